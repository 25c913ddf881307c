// Auxiliary sm_100a kernels of the int4 path: bit-exact dequant (debug
// export), device-side packer, the fp32 -> 16-bit operand cast with per-row
// power-of-two exponents, per-column scale exponents, the LoRA projection
// T = X*A, the legacy hidden-64 LoRA delta kernel, and the re-layout of
// all-gathered column shards into row-major Y.
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
    // the GEMM that follows may start its prologue (weight loads, dequant)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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

template <typename T16>
__device__ __forceinline__ uint2 pack4_16(float4 v, float scale) {
    if constexpr (std::is_same<T16, __half>::value) {
        __half2 a = __floats2half2_rn(v.x * scale, v.y * scale);
        __half2 b = __floats2half2_rn(v.z * scale, v.w * scale);
        return make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
    } else {
        __nv_bfloat162 a = __floats2bfloat162_rn(v.x * scale, v.y * scale);
        __nv_bfloat162 b = __floats2bfloat162_rn(v.z * scale, v.w * scale);
        return make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
    }
}

// The same cast for K <= 1024 R: the row is read once into registers (R
// float4 per thread, all loads in flight together), reduced, scaled and
// written; the two-pass kernel above reads it twice.
template <typename T16, int R>
__global__ void __launch_bounds__(256) cast_x_reg_kernel(const float* __restrict__ x, T16* __restrict__ x16,
                                                         int* __restrict__ row_exp, int K) {
    __shared__ float red[32];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int m = blockIdx.x;
    const float* row = x + static_cast<size_t>(m) * K;
    float4 v[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int k = (r * 256 + static_cast<int>(threadIdx.x)) * 4;
        v[r] = k < K ? __ldcs(reinterpret_cast<const float4*>(row + k)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    float scale = 1.0f;
    if (row_exp != nullptr) {
        float mx = 0.0f;
#pragma unroll
        for (int r = 0; r < R; ++r)
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[r].x), fabsf(v[r].y)), fmaxf(fabsf(v[r].z), fabsf(v[r].w))));
        mx = block_max(mx, red);
        const int e = pow2_exponent(mx, 14);
        if (threadIdx.x == 0) row_exp[m] = e;
        scale = exp2i(e);
    }
    T16* out = x16 + static_cast<size_t>(m) * K;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int k = (r * 256 + static_cast<int>(threadIdx.x)) * 4;
        if (k < K) *reinterpret_cast<uint2*>(out + k) = pack4_16<T16>(v[r], scale);
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

// T = X * A in fp32 (the LoRA projection, lora.py:21-23 forward).  A block
// covers 64 rows x 16 ranks x a 128-k chunk: it stages the X tile and the A
// slice in shared memory (all loads issued at once; rows padded so the reads
// below are free of bank conflicts), then thread (row group g = t / 16, k lane
// q = t % 16) accumulates rows 4g..4g+3 x 16 ranks over k = q, q + 16, ...
// (4 scalar X reads and 4 float4 A reads per 64 FMAs) and the 16 k lanes are
// summed with a butterfly reduce-scatter.  With one chunk the block writes T;
// with several it writes partial[z][M][rank] and lora_xa_sum_kernel (or, when
// the single-CTA GEMM needs its bf16 operand, lora_xa_reduce_kernel) sums
// the chunks in fixed order (deterministic).
constexpr int kXaRows = 64;
constexpr int kXaCols = 16;
constexpr int kXaChunk = 128;
constexpr int kXaXPitch = kXaChunk + 4;  // floats per staged X row
constexpr int kXaAPitch = kXaCols + 4;   // floats per staged A row
constexpr int kXaSmem = (kXaRows * kXaXPitch + kXaChunk * kXaAPitch) * 4;
__global__ void __launch_bounds__(256) lora_xa_kernel(const float* __restrict__ x, const float* __restrict__ a,
                                                      float* __restrict__ out, int M, int K, int rank, int kchunk) {
    extern __shared__ float xa_smem[];
    float* xs = xa_smem;                          // [64][kXaXPitch]
    float* as = xa_smem + kXaRows * kXaXPitch;    // [256][kXaAPitch]
    const int tid = threadIdx.x, lane = tid & 31;
    const int m0 = blockIdx.x * kXaRows, j0 = blockIdx.y * kXaCols;
    const int cols = min(kXaCols, rank - j0);
    float acc[4][kXaCols];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < kXaCols; ++j) acc[r][j] = 0.0f;
    const int g = tid >> 4, q = tid & 15;
    for (int kb = blockIdx.z * kchunk; kb < min(K, (blockIdx.z + 1) * kchunk); kb += kXaChunk) {
        const int kn = min(kXaChunk, K - kb);  // a multiple of 32 (K % 32 == 0)
        // stage X rows m0.. (zero past M) and A rows kb.. (zero past rank).
        // Aligned X goes by cp.async (16 bytes each, all of a thread's copies in
        // flight together), else by scalar loads.
        const bool xvec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && K % 4 == 0;
        for (int i = tid; i < kXaRows * (kXaChunk / 4); i += 256) {
            const int r = i / (kXaChunk / 4), c4 = (i % (kXaChunk / 4)) * 4;
            float* dst = xs + r * kXaXPitch + c4;
            if (m0 + r < M && c4 < kn) {
                const float* src = x + static_cast<size_t>(m0 + r) * K + kb + c4;
                if (xvec) {
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
                } else {
                    *reinterpret_cast<float4*>(dst) = make_float4(__ldg(src), __ldg(src + 1), __ldg(src + 2), __ldg(src + 3));
                }
            } else {
                *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        for (int i = tid; i < kXaChunk * kXaCols; i += 256) {
            const int k = i / kXaCols, j = i % kXaCols;
            as[k * kXaAPitch + j] = (k < kn && j < cols) ? __ldg(a + static_cast<size_t>(kb + k) * rank + j0 + j) : 0.0f;
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();
#pragma unroll 4
        for (int k = q; k < kXaChunk; k += 16) {
            float av[kXaCols];
#pragma unroll
            for (int j = 0; j < kXaCols; j += 4) {
                const float4 v = *reinterpret_cast<const float4*>(as + k * kXaAPitch + j);
                av[j] = v.x; av[j + 1] = v.y; av[j + 2] = v.z; av[j + 3] = v.w;
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float xv = xs[(4 * g + r) * kXaXPitch + k];
#pragma unroll
                for (int j = 0; j < kXaCols; ++j) acc[r][j] = fmaf(xv, av[j], acc[r][j]);
            }
        }
        __syncthreads();
    }
    // sum the 16 k lanes: butterfly over lane bits 8, 4, 2, 1 (within each
    // half warp), 64 values -> 4 per lane
    float v[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = acc[i / kXaCols][i % kXaCols];
#pragma unroll
    for (int half = 32, bit = 8; half >= 4; half >>= 1, bit >>= 1) {
        const bool upper = (lane & bit) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
        }
    }
    // lane holds values idx(q) .. idx(q) + 3 of the 64 (row-major 4 x 16)
    int idx = 0;
    if (q & 8) idx += 32;
    if (q & 4) idx += 16;
    if (q & 2) idx += 8;
    if (q & 1) idx += 4;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int r = (idx + e) / kXaCols, j = (idx + e) % kXaCols;
        const int m = m0 + 4 * g + r;
        if (m < M && j < cols) out[(static_cast<size_t>(blockIdx.z) * M + m) * rank + j0 + j] = v[e];
    }
}

// T[m][j] = sum over chunks z (fixed order) of partial[z][m][j], and the bf16
// A operand of the single-CTA GEMM's LoRA stages (tlo): row m holds ceil(rank/16) blocks of 64, block q = [hi(16) | lo(16) | hi(16) |
// 0(16)] of T[m][16q .. 16q+15] * 2^e_m, e_m = row_exp[m] (0 without), hi + lo
// carrying ~16 bits.
__global__ void __launch_bounds__(256) lora_xa_reduce_kernel(const float* __restrict__ partial,
                                                             float* __restrict__ t, int M, int rank, int chunks,
                                                             const int* __restrict__ row_exp,
                                                             __nv_bfloat16* __restrict__ tlo) {
    // one thread per (row, position) of the bf16 operand
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int W = (rank + 15) / 16 * 64;
    if (i >= M * W) return;
    const int m = i / W, pq = i % W, p = pq % 64, j = (pq / 64) * 16 + p % 16;
    float v = 0.0f;
    if (p < 48 && j < rank) {
        const int MR = M * rank;
        for (int z = 0; z < chunks; ++z) v += partial[static_cast<size_t>(z) * MR + m * rank + j];
        if (p < 16) t[m * rank + j] = v;
        v *= exp2i(row_exp != nullptr ? row_exp[m] : 0);
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        v = (p >= 16 && p < 32) ? v - __bfloat162float(hi) : __bfloat162float(hi);
    }
    tlo[i] = __float2bfloat16_rn(v);
}

// T = sum over chunks of partial[z][M * rank] for 32 outputs per CTA: warp g
// sums chunks g, g + 8, g + 16, ... in order, then one warp adds the eight
// partial sums in order (deterministic, 8x the loads in flight of one
// thread per output).
__global__ void __launch_bounds__(256) lora_xa_sum_kernel(const float* __restrict__ partial, float* __restrict__ t,
                                                          int MR, int chunks) {
    __shared__ float ps[8][32];
    const int g = threadIdx.x >> 5, o = threadIdx.x & 31;
    const int i = blockIdx.x * 32 + o;
    float s = 0.0f;
    if (i < MR)
        for (int z = g; z < chunks; z += 8) s += partial[static_cast<size_t>(z) * MR + i];
    ps[g][o] = s;
    __syncthreads();
    if (g == 0 && i < MR) {
        float v = ps[0][o];
#pragma unroll
        for (int q = 1; q < 8; ++q) v += ps[q][o];
        t[i] = v;
    }
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

namespace {
template <typename T16>
void launch_cast_t(const float* x, T16* x16, int* row_exp, int M, int K, cudaStream_t stream) {
    if (K <= 1024 * 4)
        cast_x_reg_kernel<T16, 4><<<M, 256, 0, stream>>>(x, x16, row_exp, K);
    else if (K <= 1024 * 8)
        cast_x_reg_kernel<T16, 8><<<M, 256, 0, stream>>>(x, x16, row_exp, K);
    else
        cast_x_kernel<T16><<<M, 256, 0, stream>>>(x, x16, row_exp, K);
}
}  // namespace

int launch_cast_x(const float* x, void* x16, int* row_exp, int M, int K, Operand16 op, cudaStream_t stream) {
    if (op == Operand16::kF16)
        launch_cast_t(x, static_cast<__half*>(x16), row_exp, M, K, stream);
    else
        launch_cast_t(x, static_cast<__nv_bfloat16*>(x16), row_exp, M, K, stream);
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

namespace {

// Y[m][n] += s * sum_j T[m][j] B[j][n], the LoRA term of a split-K GEMM whose
// K halves left it out (the term is then added once, after both halves, in
// the same fp32 form as the GEMM epilogue's: d = sum over j in order, y += s d).
// Block (x, m): row m, columns [1024 x, 1024 x + 1024), four per thread.
__global__ void __launch_bounds__(256) lora_add_kernel(const float* __restrict__ t, const float* __restrict__ b,
                                                       float* __restrict__ y, int N, long long ld, int rank, float s,
                                                       int vec4) {
    __shared__ float ts[64];
    const int m = blockIdx.y;
    if (threadIdx.x < rank) ts[threadIdx.x] = t[static_cast<size_t>(m) * rank + threadIdx.x];
    __syncthreads();
    const int n0 = blockIdx.x * 1024 + threadIdx.x * 4;
    float* yr = y + static_cast<size_t>(m) * ld;
    if (vec4 && n0 + 4 <= N) {
        float4 d = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int j = 0; j < rank; ++j) {
            const float4 bv = *reinterpret_cast<const float4*>(b + static_cast<size_t>(j) * N + n0);
            d.x = fmaf(ts[j], bv.x, d.x);
            d.y = fmaf(ts[j], bv.y, d.y);
            d.z = fmaf(ts[j], bv.z, d.z);
            d.w = fmaf(ts[j], bv.w, d.w);
        }
        float4 v = *reinterpret_cast<float4*>(yr + n0);
        v.x = fmaf(s, d.x, v.x);
        v.y = fmaf(s, d.y, v.y);
        v.z = fmaf(s, d.z, v.z);
        v.w = fmaf(s, d.w, v.w);
        *reinterpret_cast<float4*>(yr + n0) = v;
    } else {
        for (int n = n0; n < n0 + 4 && n < N; ++n) {
            float d = 0.0f;
            for (int j = 0; j < rank; ++j) d = fmaf(ts[j], b[static_cast<size_t>(j) * N + n], d);
            yr[n] = fmaf(s, d, yr[n]);
        }
    }
}

}  // namespace

int launch_lora_add(const float* t, const float* b, float* y, int M, int N, long long ld, int rank, float s,
                    cudaStream_t stream) {
    if (M < 1 || N < 1 || rank < 1 || rank > 64 || ld < N) return static_cast<int>(cudaErrorInvalidValue);
    const bool vec4 = N % 4 == 0 && ld % 4 == 0 && (reinterpret_cast<uintptr_t>(b) & 15u) == 0 &&
                      (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
    const dim3 grid(static_cast<unsigned>((N + 1023) / 1024), static_cast<unsigned>(M));
    lora_add_kernel<<<grid, 256, 0, stream>>>(t, b, y, N, ld, rank, s, vec4 ? 1 : 0);
    return static_cast<int>(cudaGetLastError());
}

int lora_xa_chunks(int K) { return (K + kXaChunk - 1) / kXaChunk; }

int launch_lora_xa(const float* x, const float* a, float* t, int M, int K, int rank, cudaStream_t stream,
                   float* partial, const int* row_exp, uint16_t* t_op_bits) {
    __nv_bfloat16* t_op = reinterpret_cast<__nv_bfloat16*>(t_op_bits);
    const int chunks = partial != nullptr ? lora_xa_chunks(K) : 1;
    const dim3 grid((M + kXaRows - 1) / kXaRows, (rank + kXaCols - 1) / kXaCols, chunks);
    const cudaError_t attr_ok = cudaFuncSetAttribute(lora_xa_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kXaSmem);
    if (attr_ok != cudaSuccess) return static_cast<int>(attr_ok);
    lora_xa_kernel<<<grid, 256, kXaSmem, stream>>>(x, a, chunks > 1 ? partial : t, M, K, rank,
                                                   chunks > 1 ? kXaChunk : K);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || chunks == 1) return static_cast<int>(e);
    if (t_op != nullptr) {
        const int W = (rank + 15) / 16 * 64;
        lora_xa_reduce_kernel<<<(M * W + 255) / 256, 256, 0, stream>>>(partial, t, M, rank, chunks, row_exp, t_op);
    } else {
        lora_xa_sum_kernel<<<(M * rank + 31) / 32, 256, 0, stream>>>(partial, t, M * rank, chunks);
    }
    return static_cast<int>(cudaGetLastError());
}

namespace {

// Gathered column shards [P][rows][w] (rank-major, as an all-gather of the
// per-rank Y shards leaves them) -> Y rows [rows][ld], columns [0, n_total).
// Source index order: consecutive threads read consecutive elements of one
// shard row and write consecutive columns of one Y row, so both sides
// coalesce.  V = 4 moves float4 (every address and extent 16-byte aligned),
// V = 1 single floats.
template <int V>
__global__ void __launch_bounds__(256) shards_relayout_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                              int rows, int wv, int nv, long long ldv,
                                                              long long total) {
    using T = typename std::conditional<V == 4, float4, float>::type;
    const T* s = reinterpret_cast<const T*>(src);
    T* d = reinterpret_cast<T*>(dst);
    const long long per_part = static_cast<long long>(rows) * wv;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int p = static_cast<int>(i / per_part);
        const long long rem = i - p * per_part;
        const int r = static_cast<int>(rem / wv);
        const int j = static_cast<int>(rem - static_cast<long long>(r) * wv);
        const int col = p * wv + j;
        if (col >= nv) continue;
        T v;
        if constexpr (V == 4) {
            const uint4 u = ldg_stream_v4(s + i);
            v = make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w));
        } else {
            v = __ldg(s + i);
        }
        d[r * ldv + col] = v;
    }
}

}  // namespace

int launch_shards_relayout(const float* gathered, float* y, int parts, int rows, int width, int n_total,
                           long long ld_y, cudaStream_t stream) {
    if (parts < 1 || rows < 0 || width < 1 || n_total < 1 || n_total > static_cast<long long>(parts) * width ||
        ld_y < n_total)
        return static_cast<int>(cudaErrorInvalidValue);
    if (rows == 0) return 0;
    const bool v4 = width % 4 == 0 && n_total % 4 == 0 && ld_y % 4 == 0 &&
                    (reinterpret_cast<uintptr_t>(gathered) & 15u) == 0 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
    const int v = v4 ? 4 : 1;
    const long long total = static_cast<long long>(parts) * rows * (width / v);
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long want = (total + 255) / 256;
    const unsigned grid = static_cast<unsigned>(want < 8LL * sms ? want : 8LL * sms);
    if (v4)
        shards_relayout_kernel<4><<<grid, 256, 0, stream>>>(gathered, y, rows, width / 4, n_total / 4, ld_y / 4, total);
    else
        shards_relayout_kernel<1><<<grid, 256, 0, stream>>>(gathered, y, rows, width, n_total, ld_y, total);
    return static_cast<int>(cudaGetLastError());
}

namespace {

// Rows [0, rows) x columns [0, width) of a pitched fp32 block on this GPU,
// stored to the same place in up to kMaxPeers peers' buffers (plain global
// stores through NVLink peer mappings).  Each element is read once (the band
// was just written, so mostly from L2) and stored once per peer.  A thread
// loads kPushUnroll elements (grid-stride apart) before it stores any, so a
// CTA keeps that many loads in flight instead of waiting out one load
// latency per element.  V = 4: float4 (16-byte aligned addresses, width and
// ld multiples of 4).
constexpr int kPushUnroll = 4;

template <int V>
__global__ void __launch_bounds__(512) push_rows_kernel(const float* __restrict__ src, PeerPtrs dst, int npeers,
                                                        int rows, int wv, long long ldv) {
    using T = typename std::conditional<V == 4, float4, float>::type;
    const T* s = reinterpret_cast<const T*>(src);
    const long long total = static_cast<long long>(rows) * wv;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long base = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; base < total;
         base += kPushUnroll * stride) {
        T v[kPushUnroll];
        long long at[kPushUnroll];
#pragma unroll
        for (int u = 0; u < kPushUnroll; ++u) {
            const long long i = base + u * stride;
            at[u] = -1;
            if (i < total) {
                const long long r = i / wv;
                at[u] = r * ldv + (i - r * wv);
                v[u] = s[at[u]];
            }
        }
        for (int q = 0; q < npeers; ++q) {
            T* d = reinterpret_cast<T*>(dst.p[q]);
#pragma unroll
            for (int u = 0; u < kPushUnroll; ++u)
                if (at[u] >= 0) d[at[u]] = v[u];
        }
    }
}

}  // namespace

int launch_push_rows(const float* src, const PeerPtrs& peers, int npeers, int rows, int width, long long ld, int ctas,
                     cudaStream_t stream) {
    if (npeers < 0 || npeers > kMaxPeers || rows < 0 || width < 1 || ld < width || ctas < 1)
        return static_cast<int>(cudaErrorInvalidValue);
    if (npeers == 0 || rows == 0) return 0;
    bool v4 = width % 4 == 0 && ld % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
    for (int q = 0; q < npeers; ++q) v4 = v4 && (reinterpret_cast<uintptr_t>(peers.p[q]) & 15u) == 0;
    if (v4)
        push_rows_kernel<4><<<ctas, 512, 0, stream>>>(src, peers, npeers, rows, width / 4, ld / 4);
    else
        push_rows_kernel<1><<<ctas, 512, 0, stream>>>(src, peers, npeers, rows, width, ld);
    return static_cast<int>(cudaGetLastError());
}

namespace {

// n floats from src to dst (device memory or mapped pinned host memory on
// either side), and, when status_src is given, the status word too.  A kernel
// instead of a copy-engine transfer: for the few kilobytes of a decode call's
// X and Y, the fixed cost of a copy-engine operation dominates.
// Launched as a programmatic dependent: it lets its own dependents launch at
// once (a GEMV after a copy-in starts streaming its weights while X arrives)
// and waits for its predecessor's writes (a copy-out reads the GEMV's Y).
// With done_flag (a mapped host word) the last CTA to finish publishes the
// status word and then sets done_flag to 1, after every CTA's stores are
// visible to the host: the host can wait on that word instead of a stream
// synchronisation.  done_count is a device counter that is 0 between launches.
__global__ void __launch_bounds__(256) copy_words_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                         long long n, int vec, const int* __restrict__ status_src,
                                                         int* __restrict__ status_dst, int* done_flag,
                                                         unsigned* done_count) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const long long i0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    if (vec) {
        const float4* s4 = reinterpret_cast<const float4*>(src);
        float4* d4 = reinterpret_cast<float4*>(dst);
        for (long long i = i0; i < n / 4; i += stride) d4[i] = s4[i];
    } else {
        for (long long i = i0; i < n; i += stride) dst[i] = src[i];
    }
    if (done_flag == nullptr) {
        if (status_src != nullptr && i0 == 0) *status_dst = *status_src;
        return;
    }
    // Release at device scope per CTA; the last CTA acquires every CTA's
    // stores through the counter and orders them (cumulatively) before the
    // completion word with one system-scope fence.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(done_count, 1u) == gridDim.x - 1) {
        __threadfence();
        if (status_src != nullptr) *status_dst = *status_src;
        *done_count = 0;
        __threadfence_system();
        *reinterpret_cast<volatile int*>(done_flag) = 1;
    }
}

}  // namespace

int launch_copy_words(const float* src, float* dst, long long n, const int* status_src, int* status_dst,
                      cudaStream_t stream, int* done_flag, unsigned* done_count) {
    if (n < 0 || (n > 0 && (src == nullptr || dst == nullptr)) || ((status_src == nullptr) != (status_dst == nullptr)) ||
        ((done_flag == nullptr) != (done_count == nullptr)))
        return static_cast<int>(cudaErrorInvalidValue);
    const int vec = n % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0 &&
                    (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
    const long long units = vec ? n / 4 : n;
    long long blocks = (units + 255) / 256;
    if (blocks < 1) blocks = 1;
    if (blocks > 1024) blocks = 1024;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(blocks));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return static_cast<int>(
        cudaLaunchKernelEx(&cfg, copy_words_kernel, src, dst, n, vec, status_src, status_dst, done_flag, done_count));
}

int launch_lora_delta64(const float* x, const float* a, const float* b, float* y, int M, int rank,
                        cudaStream_t stream) {
    lora_delta64_kernel<<<M, 64, 0, stream>>>(x, a, b, y, rank);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace q4
