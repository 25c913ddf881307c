// Decode GEMV (M <= 8):  Y[M x N] = X[M x K] . dequant(W)  (+ LoRA term), fp32.
//
// Replaces the decode use of vulkan-runtime/shaders/q4gemm.comp:61-175 (the
// reference kernel itself needs M % 64 == 0, q4gemm.comp:36-37, so it has no
// decode path).  Same weight layout (q4gemm.comp:7-19):
//   packed byte pb = n*(K/2) + k/2, low nibble = even k, v & 0xF two's complement;
//   scale (k, n) = scales[n*(K/32) + k/32];  w = float(v) * scale.
// Because K % 32 == 0, the 16 bytes of one column's 32-k scale group are one
// aligned 128-bit word.
//
// Structure (HBM streaming, one CTA per SM):
//   * a cluster of S CTAs splits K into S slices of GS <= 32 scale groups;
//     the cluster owns a contiguous column range;
//   * a producer warp streams the cluster range's packed weights (2-D TMA,
//     CC columns x the slice's bytes per chunk) and scales (4-byte cp.async,
//     zero-filled outside the matrix) for this CTA's K slice into a
//     shared-memory ring, starting before griddepcontrol.wait, so under
//     programmatic dependent launch the weights of this launch stream in while
//     the previous launch drains;
//   * 8 consumer warps: lane l owns scale group l of the slice and keeps that
//     group's 32 x values (up to 4 rows) in registers for the whole kernel;
//     per column it reads one 16-byte word (32 nibbles) and one scale from
//     shared memory, forms sum_j x_j * v_j exactly-unpacked in fp32, scales
//     once per group, and the warp reduce-scatters its CW columns x rows
//     partials across lanes with a butterfly (V-1+5-log2 V shuffles);
//   * the K-slice partials are summed across the cluster through distributed
//     shared memory in fixed rank order (deterministic, no atomics, no global
//     scratch), the optional LoRA term (alpha/r) * T[m,:] . B[:, n] with
//     T = X*A is added and Y is stored.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "q4_kernels.h"

namespace cg = cooperative_groups;

namespace q4 {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;  // + 1 producer warp
constexpr int kCW = 2;                                   // columns per warp per chunk
constexpr int kCC = kConsumerWarps * kCW;                // columns per chunk (16)
constexpr int kStages = 4;

// Exact unpack of one packed word (8 nibbles, k = 0..7 at bits 4k) to floats
// with the 2^23 magic number: (u ^ 8) = v + 8 in [0, 15], and
// float(0x4B000000 | (v + 8)) = 2^23 + v + 8.
__device__ __forceinline__ void unpack8(uint32_t q, float (&v)[8]) {
    const uint32_t lo = (q ^ 0x88888888u) & 0x0F0F0F0Fu;         // k = 0, 2, 4, 6
    const uint32_t hi = ((q >> 4) ^ 0x08080808u) & 0x0F0F0F0Fu;  // k = 1, 3, 5, 7
    const float bias = 8388616.0f;                                // 2^23 + 8
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        // byte_perm selector 0x744b: byte b of the word -> byte 0, zero bytes
        // -> bytes 1-2, 0x4B (the exponent byte of 2^23) -> byte 3.
        v[2 * b] = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b))) - bias;
        v[2 * b + 1] = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b))) - bias;
    }
}

// X slice in shared memory: [group][k in group 0..31][row m] (M floats per k),
// float4 units of a group XOR-swizzled with (group & 7) so the 8 lanes of a
// quarter warp, reading the same unit of 8 different groups, hit 8 different
// bank quads.
template <int M>
__device__ __forceinline__ int xs_offset(int g, int unit) {
    return g * (32 * M) + ((unit ^ (g & 7)) << 2);
}

template <int M>
struct GemvCfg {
    static constexpr int MR = M < 4 ? M : 4;           // rows per register pass
    static constexpr int kPasses = (M + MR - 1) / MR;  // 1 or 2
    static constexpr int V = kCW * (MR == 3 ? 4 : MR); // reduce-scatter width (power of 2)
};

struct GemvSmem {
    int GS, GSp;               // groups in the slice; scale row pitch in the ring
    int w_bytes, s_bytes;      // per stage
    int stage_bytes;
    int xs_floats;
    int part_floats;
};

__host__ __device__ inline GemvSmem gemv_layout(int M, int K, int S, int cols_per_cluster) {
    GemvSmem L;
    L.GS = K / 32 / S;
    L.GSp = L.GS;
    L.w_bytes = kCC * L.GS * 16;
    L.s_bytes = kCC * L.GSp * 4;
    L.stage_bytes = L.w_bytes + L.s_bytes;
    L.xs_floats = L.GS * 32 * M;
    L.part_floats = cols_per_cluster * M;
    return L;
}

// Test hook (gemv_ring_set_wait_test): when set, consumer warp 0 of every
// CTA first waits for the second phase of ring stage 0's barrier, which the
// producer cannot arm before that warp releases the stage, so the bounded
// wait runs out and the timeout path runs.  Read once per thread at entry.
static __device__ int g_ring_stall_test = 0;

template <int M>
__global__ void __launch_bounds__(kGemvThreads, 1)
    q4_gemv_kernel(const __grid_constant__ CUtensorMap tmap_w, const float* __restrict__ scales,
                   const float* __restrict__ x, float* __restrict__ y, int N, int K, int cols_per_cluster,
                   const float* __restrict__ lora_t, const float* __restrict__ lora_b, int rank,
                   float lora_scale, int* __restrict__ status) {
    using C = GemvCfg<M>;
    extern __shared__ __align__(128) uint8_t smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const int S = static_cast<int>(cluster.num_blocks());
    const int rank_k = static_cast<int>(cluster.block_rank());
    const int cluster_id = blockIdx.x / S;
    const GemvSmem L = gemv_layout(M, K, S, cols_per_cluster);
    const int GS = L.GS;
    const int g0 = rank_k * GS;                // first group of this K slice
    const int n0 = cluster_id * cols_per_cluster;
    const int ncols = max(0, min(N, n0 + cols_per_cluster) - n0);
    const int nchunks = (ncols + kCC - 1) / kCC;

    uint8_t* stage_base = smem;
    float* xs = reinterpret_cast<float*>(smem + kStages * L.stage_bytes);
    float* part = xs + L.xs_floats;
    uint64_t* bars = reinterpret_cast<uint64_t*>(part + L.part_floats + ((L.part_floats & 1) ? 1 : 0));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * kStages);
    auto full = [&](int s) { return smem_u32(bars + s); };
    auto empty = [&](int s) { return smem_u32(bars + kStages + s); };

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int stall_test = warp == 0 ? *static_cast<volatile int*>(&g_ring_stall_test) : 0;
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full(s), 1 + 32);  // TMA expect_tx arrival + 32 producer cp.async arrivals
            mbar_init(empty(s), kConsumerWarps);
        }
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    __syncthreads();

    const int G = K / 32;
    // Producer warp, all lanes: chunk j -> ring stage j % kStages.  Lane 0
    // issues the weight TMA (expect_tx), every lane copies its share of the
    // chunk's scales with cp.async and arrives once those land.
    auto issue = [&](int j) {
        const int s = j % kStages;
        const uint32_t dst = smem_u32(stage_base + s * L.stage_bytes);
        if (lane == 0) {
            mbar_arrive_expect_tx(full(s), static_cast<uint32_t>(L.w_bytes));
            tma_load_2d(dst, &tmap_w, full(s), g0 * 4, n0 + j * kCC);
        }
        const uint32_t sdst = dst + L.w_bytes;
        for (int e = lane; e < kCC * GS; e += 32) {
            const int cl = e / GS, gg = e % GS;
            const int n = n0 + j * kCC + cl;
            const bool ok = n < N;
            const float* src = scales + (static_cast<size_t>(ok ? n : 0) * G + g0 + gg);
            cp_async4(sdst + e * 4, src, ok ? 4u : 0u);
        }
        cp_async_arrive_noinc(full(s));
    };
    int issued = 0;
    if (warp == kConsumerWarps) {
        if (lane == 0) tma_prefetch_desc(&tmap_w);
        // Weights and scales do not depend on the previous launch: the first
        // ring's worth streams in before griddepcontrol.wait.
        for (; issued < nchunks && issued < kStages; ++issued) issue(issued);
    }
    pdl_wait();  // X (and LoRA T) may be written by the previous launch
    if (warp < kConsumerWarps) {
        // Stage this CTA's slice of X: rows 0..M-1, k in [g0*32, g0*32 + 32*GS).
        for (int idx = tid; idx < GS * 8 * M; idx += kConsumerWarps * 32) {
            const int g = idx / (8 * M), unit = idx % (8 * M);
            float t[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int flat = unit * 4 + e;  // = j*M + m
                t[e] = x[static_cast<size_t>(flat % M) * K + (g0 + g) * 32 + flat / M];
            }
            *reinterpret_cast<float4*>(xs + xs_offset<M>(g, unit)) = make_float4(t[0], t[1], t[2], t[3]);
        }
    }
    __syncthreads();
    // Dependent launches may start their prologue (their own weight stream).
    pdl_launch_dependents();

    if (warp == kConsumerWarps) {
        // ------------------------------------------- producer: refill ring --
        for (; issued < nchunks; ++issued) {
            const int j = issued;
            if (!mbar_wait(empty(j % kStages), ((j / kStages) - 1) & 1u, abort_flag, status, kStatusTimeoutGemv))
                break;
            issue(j);
        }
    }
    if (warp < kConsumerWarps) {
        // ---------------------------------------------------- consumers --
        const bool active = lane < GS;
        const int g = active ? lane : 0;
        float xr[32][C::MR];
        // This lane's 32 x values for rows mbase .. mbase+MR-1.
        auto load_x = [&](int mbase) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
#pragma unroll
                for (int r = 0; r < C::MR; ++r) {
                    const int m = mbase + r;
                    const int flat = j * M + (m < M ? m : 0);
                    const float v = xs[xs_offset<M>(g, flat >> 2) + (flat & 3)];
                    xr[j][r] = (active && m < M) ? v : 0.0f;
                }
        };
        if (C::kPasses == 1) load_x(0);
        bool stalled = false;
        if (stall_test)  // phase 0 of stage 0 completes; its phase 1 waits on this warp
            stalled = !(mbar_wait(full(0), 0u, abort_flag, status, kStatusTimeoutGemv) &&
                        mbar_wait(full(0), 1u, abort_flag, status, kStatusTimeoutGemv));
        for (int jc = 0; jc < nchunks && !stalled; ++jc) {
            const int s = jc % kStages;
            if (!mbar_wait(full(s), (jc / kStages) & 1u, abort_flag, status, kStatusTimeoutGemv)) break;
            const uint8_t* wst = stage_base + s * L.stage_bytes;
            const float* sst = reinterpret_cast<const float*>(wst + L.w_bytes);
#pragma unroll 1
            for (int pass = 0; pass < C::kPasses; ++pass) {
                const int mbase = pass * C::MR;
                if (C::kPasses > 1) load_x(mbase);
                float acc[C::V];
#pragma unroll
                for (int i = 0; i < C::V; ++i) acc[i] = 0.0f;
                constexpr int RP = C::V / kCW;  // row slots per column (power of two)
#pragma unroll
                for (int c = 0; c < kCW; ++c) {
                    const int cl = warp * kCW + c;  // column inside the chunk
                    const uint4 q = *reinterpret_cast<const uint4*>(wst + (cl * GS + g) * 16);
                    const float sc = active ? sst[cl * L.GSp + g] : 0.0f;
                    float gacc[C::MR];
#pragma unroll
                    for (int r = 0; r < C::MR; ++r) gacc[r] = 0.0f;
                    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int wd = 0; wd < 4; ++wd) {
                        float v[8];
                        unpack8(words[wd], v);
#pragma unroll
                        for (int i = 0; i < 8; ++i)
#pragma unroll
                            for (int r = 0; r < C::MR; ++r) gacc[r] = fmaf(xr[wd * 8 + i][r], v[i], gacc[r]);
                    }
#pragma unroll
                    for (int r = 0; r < C::MR; ++r) acc[c * RP + r] = sc * gacc[r];
                }
                const float red = warp_reduce_scatter<C::V>(acc, lane);
                const int idx = value_index<C::V>(lane);
                const int c = idx / RP, r = idx % RP;
                const int col = jc * kCC + warp * kCW + c;
                const int m = mbase + r;
                // Each value is held by 32/V lanes; the lowest one writes.
                const bool writer = (lane & ((32 / C::V) - 1)) == 0;
                if (writer && r < C::MR && m < M && col < ncols) part[col * M + m] = red;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty(s));
        }
    }

    if (warp == kConsumerWarps && *abort_flag) {
        // Abort path: let this CTA's copies in flight land before it exits.
        cp_async_wait_all();
        if (lane == 0)
            for (int j = (issued > kStages ? issued - kStages : 0); j < issued; ++j)
                mbar_drain(full(j % kStages), (j / kStages) & 1u);
    }

    // Cross-slice reduction through distributed shared memory, fixed order.
    cluster.sync();
    if (*abort_flag == 0) {
        for (int idx = tid; idx < ncols * M; idx += kGemvThreads) {
            const int lc = idx / M, m = idx % M;
            if (lc % S != rank_k) continue;  // columns interleaved over the cluster's CTAs
            float sum = 0.0f;
            for (int r = 0; r < S; ++r) sum += cluster.map_shared_rank(part, r)[idx];
            const int n = n0 + lc;
            if (lora_t != nullptr) {
                float d = 0.0f;
                for (int j = 0; j < rank; ++j)
                    d = fmaf(lora_t[m * rank + j], lora_b[static_cast<size_t>(j) * N + n], d);
                sum = fmaf(lora_scale, d, sum);
            }
            y[static_cast<size_t>(m) * N + n] = sum;
        }
    }
    cluster.sync();  // keep this CTA's partials alive until every peer has read them
}

size_t smem_bytes_for(int M, int K, int S, int cols_per_cluster) {
    const GemvSmem L = gemv_layout(M, K, S, cols_per_cluster);
    return static_cast<size_t>(kStages) * L.stage_bytes + (L.xs_floats + L.part_floats + 1) * 4 + 2 * kStages * 8 +
           16;
}

template <int M>
int max_clusters_m(int K, int S, int cols_per_cluster) {
    const size_t smem = smem_bytes_for(M, K, S, cols_per_cluster);
    auto kern = q4_gemv_kernel<M>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
        return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(S), 1, 1);
    cfg.blockDim = dim3(kGemvThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(S);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) return 0;
    return n;
}

template <int M>
int launch_gemv_m(const GemvArgs& a, cudaStream_t stream) {
    const int S = a.cluster_k;
    const size_t smem = smem_bytes_for(M, a.K, S, a.cols_per_cluster);
    auto kern = q4_gemv_kernel<M>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(S * a.clusters), 1, 1);
    cfg.blockDim = dim3(kGemvThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(S);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, kern, a.tmap_w, a.scales, a.x, a.y, a.N, a.K, a.cols_per_cluster, a.lora_t,
                           a.lora_b, a.rank, a.lora_scale, a.status);
    return static_cast<int>(e);
}

}  // namespace

size_t gemv_smem_bytes(int M, int K, int cluster_k, int cols_per_cluster) {
    return smem_bytes_for(M, K, cluster_k, cols_per_cluster);
}

int gemv_max_active_clusters(int M, int K, int cluster_k, int cols_per_cluster) {
    switch (M) {
        case 1: return max_clusters_m<1>(K, cluster_k, cols_per_cluster);
        case 2: return max_clusters_m<2>(K, cluster_k, cols_per_cluster);
        case 3: return max_clusters_m<3>(K, cluster_k, cols_per_cluster);
        case 4: return max_clusters_m<4>(K, cluster_k, cols_per_cluster);
        case 5: return max_clusters_m<5>(K, cluster_k, cols_per_cluster);
        case 6: return max_clusters_m<6>(K, cluster_k, cols_per_cluster);
        case 7: return max_clusters_m<7>(K, cluster_k, cols_per_cluster);
        case 8: return max_clusters_m<8>(K, cluster_k, cols_per_cluster);
        default: return 0;
    }
}

int gemv_chunk_columns() { return kCC; }

int gemv_ring_set_wait_test(unsigned long long limit_ns, int stall) {
    cudaError_t e = cudaMemcpyToSymbol(g_wait_limit_ns, &limit_ns, sizeof(limit_ns));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_ring_stall_test, &stall, sizeof(stall));
    return static_cast<int>(e);
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
