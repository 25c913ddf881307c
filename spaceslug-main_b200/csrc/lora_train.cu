// LoRA training around the fused forward Y = X * dequant(W) + s * (X * A) * B
// (s = alpha / rank; W frozen): the adapter gradients and the optimiser
// updates.
//
//   dB[r][N] = s * T^T * dY      with T = X * A      [M x r]
//   dA[K][r] = s * X^T * G       with G = dY * B^T   [M x r]
//
// the reference's lora_gradients (vulkan-runtime/src/api/lora_gradients_api.h:4-6:
// dA = X^T dY B^T, dB = (X A)^T dY, s = 1 there) generalised to any K, N and
// rank <= 64.  T and G reuse the split-K projection kernels of q4_aux.cu (G
// with B^T materialised by transpose_kernel).  The two "outer" products reduce
// over the M rows: outer_partial_kernel gives one partial per 64-row chunk
// (thread = one column c, 16 ranks of accumulators, the chunk's 64 x 16 left
// factor staged in shared memory) and outer_reduce_kernel sums the partials in
// chunk order (deterministic), scales by s and writes either [r][C] (dB) or
// [C][r] (dA).  sgd_kernel / adamw_kernel update a parameter array in place.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "q4_kernels.h"

namespace q4 {

namespace {

constexpr int kOuterRows = 64;   // rows of M per partial
constexpr int kOuterRanks = 16;  // ranks per thread
constexpr int kOuterCols = 256;  // columns per CTA (one per thread)

__global__ void __launch_bounds__(256) transpose_kernel(const float* __restrict__ b, float* __restrict__ bt, int rank,
                                                        int N) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<long long>(rank) * N) return;
    const int j = static_cast<int>(i / N), n = static_cast<int>(i % N);
    bt[static_cast<size_t>(n) * rank + j] = b[i];
}

// partial[z][j][c] = sum over rows m of chunk z of L[m][j] * R[m][c]
__global__ void __launch_bounds__(kOuterCols) outer_partial_kernel(const float* __restrict__ L,
                                                                   const float* __restrict__ R,
                                                                   float* __restrict__ partial, int M, int rank,
                                                                   int C) {
    __shared__ float ls[kOuterRows][kOuterRanks];
    const int c = blockIdx.x * kOuterCols + threadIdx.x;
    const int j0 = blockIdx.y * kOuterRanks;
    const int m0 = blockIdx.z * kOuterRows;
    const int rows = min(kOuterRows, M - m0);
    for (int i = threadIdx.x; i < kOuterRows * kOuterRanks; i += blockDim.x) {
        const int mm = i / kOuterRanks, jj = i % kOuterRanks;
        ls[mm][jj] = (mm < rows && j0 + jj < rank) ? L[static_cast<size_t>(m0 + mm) * rank + j0 + jj] : 0.0f;
    }
    __syncthreads();
    if (c >= C) return;
    float acc[kOuterRanks];
#pragma unroll
    for (int j = 0; j < kOuterRanks; ++j) acc[j] = 0.0f;
    for (int mm = 0; mm < rows; ++mm) {
        const float r = R[static_cast<size_t>(m0 + mm) * C + c];
#pragma unroll
        for (int j = 0; j < kOuterRanks; ++j) acc[j] = fmaf(ls[mm][j], r, acc[j]);
    }
    float* out = partial + static_cast<size_t>(blockIdx.z) * rank * C;
#pragma unroll
    for (int j = 0; j < kOuterRanks; ++j)
        if (j0 + j < rank) out[static_cast<size_t>(j0 + j) * C + c] = acc[j];
}

// out = s * sum_z partial[z]; transpose_out: out[c][j] (K x r), else out[j][c] (r x C).
__global__ void __launch_bounds__(256) outer_reduce_kernel(const float* __restrict__ partial, float* __restrict__ out,
                                                           int chunks, int rank, int C, float s, int transpose_out) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long total = static_cast<long long>(rank) * C;
    if (i >= total) return;
    float v = 0.0f;
    for (int z = 0; z < chunks; ++z) v += partial[static_cast<size_t>(z) * total + i];
    v *= s;
    const int j = static_cast<int>(i / C), c = static_cast<int>(i % C);
    if (transpose_out) out[static_cast<size_t>(c) * rank + j] = v;
    else out[i] = v;
}

__global__ void __launch_bounds__(256) sgd_kernel(float* __restrict__ p, const float* __restrict__ g, float lr,
                                                  long long count) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < count) p[i] = p[i] - lr * g[i];
}

// AdamW (decoupled weight decay), bias-corrected moments; c1 = 1 - beta1^t, c2 = 1 - beta2^t.
__global__ void __launch_bounds__(256) adamw_kernel(float* __restrict__ p, const float* __restrict__ g,
                                                    float* __restrict__ m1, float* __restrict__ m2, float lr,
                                                    float beta1, float beta2, float eps, float wd, float c1, float c2,
                                                    long long count) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const float gi = g[i];
    const float a = beta1 * m1[i] + (1.0f - beta1) * gi;
    const float b = beta2 * m2[i] + (1.0f - beta2) * gi * gi;
    m1[i] = a;
    m2[i] = b;
    const float mh = a / c1, vh = b / c2;
    p[i] = p[i] - lr * (mh / (sqrtf(vh) + eps) + wd * p[i]);
}

inline unsigned blocks(long long work, int block) { return static_cast<unsigned>((work + block - 1) / block); }

}  // namespace

size_t lora_backward_scratch_floats(int M, int K, int N, int rank) {
    const size_t chunks = static_cast<size_t>((M + kOuterRows - 1) / kOuterRows);
    const size_t cmax = static_cast<size_t>(K > N ? K : N);
    const size_t xa_part = static_cast<size_t>(lora_xa_chunks(K > N ? K : N)) * M * rank;
    // T, G, B^T, xa partials, outer partials
    return 2 * static_cast<size_t>(M) * rank + static_cast<size_t>(N) * rank + xa_part + chunks * rank * cmax;
}

int launch_lora_backward(const LoraBackwardArgs& a, cudaStream_t stream) {
    const int M = a.M, K = a.K, N = a.N, r = a.rank;
    if (M < 1 || K < 1 || N < 1 || r < 1 || r > 64) return static_cast<int>(cudaErrorInvalidValue);
    float* T = a.scratch;
    float* G = T + static_cast<size_t>(M) * r;
    float* BT = G + static_cast<size_t>(M) * r;
    float* xa_part = BT + static_cast<size_t>(N) * r;
    float* outer = xa_part + static_cast<size_t>(lora_xa_chunks(K > N ? K : N)) * M * r;
    int e;
    // T = X A, G = dY B^T
    if ((e = launch_lora_xa(a.x, a.lora_a, T, M, K, r, stream, xa_part)) != 0) return e;
    transpose_kernel<<<blocks(static_cast<long long>(r) * N, 256), 256, 0, stream>>>(a.lora_b, BT, r, N);
    if ((e = static_cast<int>(cudaGetLastError())) != 0) return e;
    if ((e = launch_lora_xa(a.dy, BT, G, M, N, r, stream, xa_part)) != 0) return e;
    const int chunks = (M + kOuterRows - 1) / kOuterRows;
    const dim3 rgrid(1, static_cast<unsigned>((r + kOuterRanks - 1) / kOuterRanks), static_cast<unsigned>(chunks));
    // dB = s T^T dY  [r][N]
    dim3 g1 = rgrid;
    g1.x = blocks(N, kOuterCols);
    outer_partial_kernel<<<g1, kOuterCols, 0, stream>>>(T, a.dy, outer, M, r, N);
    if ((e = static_cast<int>(cudaGetLastError())) != 0) return e;
    outer_reduce_kernel<<<blocks(static_cast<long long>(r) * N, 256), 256, 0, stream>>>(outer, a.db, chunks, r, N,
                                                                                         a.scale, 0);
    if ((e = static_cast<int>(cudaGetLastError())) != 0) return e;
    // dA = s X^T G  [K][r]
    dim3 g2 = rgrid;
    g2.x = blocks(K, kOuterCols);
    outer_partial_kernel<<<g2, kOuterCols, 0, stream>>>(G, a.x, outer, M, r, K);
    if ((e = static_cast<int>(cudaGetLastError())) != 0) return e;
    outer_reduce_kernel<<<blocks(static_cast<long long>(r) * K, 256), 256, 0, stream>>>(outer, a.da, chunks, r, K,
                                                                                         a.scale, 1);
    return static_cast<int>(cudaGetLastError());
}

int launch_sgd(float* p, const float* g, float lr, long long count, cudaStream_t stream) {
    if (count <= 0) return 0;
    sgd_kernel<<<blocks(count, 256), 256, 0, stream>>>(p, g, lr, count);
    return static_cast<int>(cudaGetLastError());
}

int launch_adamw(float* p, const float* g, float* m1, float* m2, float lr, float beta1, float beta2, float eps,
                 float wd, int step, long long count, cudaStream_t stream) {
    if (count <= 0) return 0;
    const float c1 = 1.0f - std::pow(beta1, static_cast<float>(step));
    const float c2 = 1.0f - std::pow(beta2, static_cast<float>(step));
    adamw_kernel<<<blocks(count, 256), 256, 0, stream>>>(p, g, m1, m2, lr, beta1, beta2, eps, wd, c1, c2, count);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace q4
