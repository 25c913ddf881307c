// Decode (M <= 8) on the tensor cores:  Y[M x N] = X . dequant(W) (+ LoRA), fp32
// accuracy.
//
// The reference has no decode path (q4gemm.comp:36-37 needs M % 64 == 0); the
// math is its dequant w = float(v) * scale (q4gemm.comp:104-122) and a dot
// product over K.  Doing that on CUDA cores costs ~2 + M instructions per
// weight, which is more than the HBM stream allows at M = 8.  Here the
// weights are the MMA's A operand and the per-group scale is applied after
// the MMA, so a weight costs ~2 instructions whatever M is:
//
//   * A = W^T tile: 128 weight columns (TMEM lanes) x 64 k, the int4 values
//     v themselves as f16 (exact), written by the dequant warps into the
//     canonical K-major 128B-swizzled layout;
//   * B = X^T: 16 "rows" = x_hi (8 rows) and x_lo (8 rows), x * 2^e = x_hi +
//     x_lo split into two f16 with a power-of-two exponent e per (row, K
//     slice); built once per CTA for its K slice (v is exact, x_hi + x_lo
//     carries ~22 bits, fp32 accumulation: the product error is ~2^-21);
//   * one tcgen05.mma pair (K = 16 x 2) per 32-k scale group writes a 128 x 16
//     fp32 partial into its own TMEM slot; four "scale" warps read the slot
//     (thread = weight column) and accumulate y[m] += s(n, g) *
//     (D[m] + D[8 + m]) in registers;
//   * the K slices of a column block run on the CTAs of a cluster (8 x 512 k
//     at K = 4096); their partials are summed through distributed shared
//     memory in fixed rank order, the LoRA term is added and Y is stored.
//
// All weight loads are issued before griddepcontrol.wait, so under
// programmatic dependent launch a launch streams its weights while the
// previous launch finishes.  No load is shared across CTAs.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "q4_dequant.cuh"
#include "q4_kernels.h"

namespace cg = cooperative_groups;

namespace q4 {

namespace {

constexpr int kCols = 128;          // weight columns per CTA (MMA M, TMEM lanes)
constexpr int kStageK = 64;         // k per stage (2 scale groups)
constexpr int kAStages = 3;         // dequantised A tiles in flight
constexpr int kSlots = 8;           // TMEM partial slots (16 columns each)
constexpr int kThreads = 320;       // 10 warps
constexpr int kDqWarp0 = 2;         // dequant warps 2..5
constexpr int kDqWarps = 4;
constexpr int kScWarp0 = 6;         // scale warps 6..9 (TMEM lane quarters 2, 3, 0, 1)
constexpr int kScWarps = 4;
constexpr int kMaxGroups = 32;      // scale groups per K slice

struct DLayout {
    int GS;           // scale groups in the slice (even, <= 32)
    int stages;       // GS / 2
    int raw_off, a_off, bx_off, part_off, bar_off, misc_off, bytes;
};

__host__ __device__ inline DLayout decode_layout(int K, int S) {
    DLayout L;
    L.GS = K / 32 / S;
    L.stages = L.GS / 2;
    L.a_off = 0;                                           // kAStages x 16 KB (1024-aligned)
    L.bx_off = L.a_off + kAStages * kCols * 128;           // stages x 2 KB (1024-aligned)
    L.raw_off = L.bx_off + L.stages * 2048;                // stages x 4 KB
    L.part_off = L.raw_off + L.stages * kCols * 32;        // 128 x 8 floats
    L.bar_off = L.part_off + kCols * 8 * 4;
    // raw_full[stages], a_full[3], a_empty[3], d_full[8], d_empty[8]
    L.misc_off = L.bar_off + (L.stages + 2 * kAStages + 2 * kSlots) * 8;
    L.bytes = L.misc_off + 16 + 8 * 4;                     // tmem holder, abort flag, row exponents
    return L;
}

// 8 int4 values of one packed word as four f16 pairs (k, k+1), exact.
__device__ __forceinline__ uint4 unpack_word_f16(uint32_t q) {
    const uint32_t lo = (q ^ 0x88888888u) & 0x0F0F0F0Fu;
    const uint32_t hi = ((q >> 4) ^ 0x08080808u) & 0x0F0F0F0Fu;
    const float2 nbias = make_float2(-8388616.0f, -8388616.0f);
    uint32_t out[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const float2 mg = make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b))),
                                      __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b))));
        const float2 v = __fadd2_rn(mg, nbias);
        out[b] = pack2<__half>(v.x, v.y);
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
}

// Power-of-two exponent e with max|x| * 2^e in [2^13, 2^14) (0 for a zero or
// non-finite maximum), so x * 2^e splits into f16 hi + lo without overflow.
__device__ __forceinline__ int row_exponent(float mx) {
    if (!(mx > 0.0f) || !isfinite(mx)) return 0;
    int e2;
    frexpf(mx, &e2);
    const int e = 14 - e2;
    return e < -60 ? -60 : (e > 60 ? 60 : e);
}

// Byte offset of (row r, k index kk in 0..63) inside one 16-row x 64-k
// K-major 128B-swizzled tile.
__device__ __forceinline__ int sw128_offset(int r, int kk) {
    return r * 128 + ((((kk >> 3) ^ (r & 7))) << 4) + (kk & 7) * 2;
}

__global__ void __launch_bounds__(kThreads, 2)
    q4_decode_kernel(const __grid_constant__ CUtensorMap tmap_w, const float* __restrict__ x,
                     const float* __restrict__ scales, float* __restrict__ y, int M, int N, int K,
                     const float* __restrict__ lora_t, const float* __restrict__ lora_b, int rank, float lora_scale,
                     int* __restrict__ status) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_base);

    cg::cluster_group cluster = cg::this_cluster();
    const int S = static_cast<int>(cluster.num_blocks());
    const int crank = static_cast<int>(cluster.block_rank());
    const DLayout L = decode_layout(K, S);
    const int GS = L.GS, NST = L.stages;
    const int G = K / 32;
    const int g0 = crank * GS;                  // first group of this K slice
    const int k0 = g0 * 32;
    const int n0 = (blockIdx.x / S) * kCols;    // the cluster's column block

    const uint32_t bar = base + L.bar_off;
    auto raw_full = [&](int st) { return bar + 8u * st; };
    auto a_full = [&](int i) { return bar + 8u * (NST + i); };
    auto a_empty = [&](int i) { return bar + 8u * (NST + kAStages + i); };
    auto d_full = [&](int i) { return bar + 8u * (NST + 2 * kAStages + i); };
    auto d_empty = [&](int i) { return bar + 8u * (NST + 2 * kAStages + kSlots + i); };
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L.misc_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off + 4);
    int* row_max = reinterpret_cast<int*>(smem + L.misc_off + 16);  // [8] max |x| of each row (float bits)
    float* part = reinterpret_cast<float*>(smem + L.part_off);      // [128][8]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int st = 0; st < NST; ++st) mbar_init(raw_full(st), 1);
        for (int i = 0; i < kAStages; ++i) {
            mbar_init(a_full(i), kDqWarps);
            mbar_init(a_empty(i), 1);
        }
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(d_full(i), 1);
            mbar_init(d_empty(i), kScWarps);
        }
        *abort_flag = 0;
        for (int m = 0; m < 8; ++m) row_max[m] = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_holder), kSlots * 16);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_holder;

    // Weights do not depend on the previous launch: the whole slice's packed
    // W streams in (one 2-D TMA box per 64-k stage) before griddepcontrol.wait.
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmap_w);
        for (int st = 0; st < NST; ++st) {
            mbar_arrive_expect_tx(raw_full(st), kCols * 32);
            tma_load_2d(base + L.raw_off + st * kCols * 32, &tmap_w, raw_full(st), (k0 + st * kStageK) / 8, n0);
        }
    }
    // Scale warps: this thread's column scales for the slice, also before the wait.
    float sc[kMaxGroups];
    const int quarter = warp & 3;
    const int col = quarter * 32 + lane;  // TMEM lane = weight column within the block
    if (warp >= kScWarp0) {
        const int n = n0 + col;
        const float* srow = scales + static_cast<size_t>(n < N ? n : 0) * G + g0;
#pragma unroll
        for (int g = 0; g < kMaxGroups; ++g) sc[g] = (g < GS && n < N) ? __ldg(srow + g) : 0.0f;
    }

    pdl_wait();  // X and the LoRA projection may come from the previous launch

    // ---------------------------------------------------- B = X^T tile --
    // Row maxima over the slice (non-negative float bits order like ints).
    if (warp >= kDqWarp0) {
        const int t = tid - kDqWarp0 * 32;  // 0..255
        for (int m = 0; m < M; ++m) {
            float mx = 0.0f;
            for (int k = t; k < GS * 32; k += 256) mx = fmaxf(mx, fabsf(x[static_cast<size_t>(m) * K + k0 + k]));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            if (lane == 0) atomicMax(&row_max[m], __float_as_int(mx));
        }
    }
    __syncthreads();
    if (warp >= kDqWarp0) {
        const int t = tid - kDqWarp0 * 32;
        // per-row exponent e with max|x * 2^e| in [2^13, 2^14)
        float rs[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) rs[m] = exp2i(row_exponent(__int_as_float(row_max[m])));
        // units: (row m of 8, 8-k chunk of the slice); writes the hi row m and
        // the lo row 8 + m of the stage tile
        const int chunks = GS * 4;
        for (int u = t; u < 8 * chunks; u += 256) {
            const int m = u / chunks, c = u % chunks;
            const int st = c / 8, kk = (c % 8) * 8;
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float a0 = 0.0f, a1 = 0.0f;
                if (m < M) {
                    a0 = x[static_cast<size_t>(m) * K + k0 + c * 8 + 2 * i] * rs[m];
                    a1 = x[static_cast<size_t>(m) * K + k0 + c * 8 + 2 * i + 1] * rs[m];
                }
                const __half2 h = __floats2half2_rn(a0, a1);
                const float2 hf = __half22float2(h);
                const __half2 l = __floats2half2_rn(a0 - hf.x, a1 - hf.y);
                hw[i] = *reinterpret_cast<const uint32_t*>(&h);
                lw[i] = *reinterpret_cast<const uint32_t*>(&l);
            }
            uint8_t* tile = smem + L.bx_off + st * 2048;
            *reinterpret_cast<uint4*>(tile + sw128_offset(m, kk)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4*>(tile + sw128_offset(8 + m, kk)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        fence_proxy_async_smem();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == 1) {
        // ------------------------------------------------------------- MMA --
        if (elect_one()) {
            const uint32_t idesc = umma_idesc_f16(0u, 128u, 16u);
            bool ok = true;
            for (int st = 0; st < NST && ok; ++st) {
                const int ai = st % kAStages;
                if (!mbar_wait(a_full(ai), (st / kAStages) & 1u, abort_flag, status, kStatusTimeoutMma)) break;
                tc_fence_after_sync();
#pragma unroll
                for (int g = 0; g < 2; ++g) {
                    const int gi = st * 2 + g, slot = gi % kSlots;
                    if (!mbar_wait(d_empty(slot), ((gi / kSlots) & 1u) ^ 1u, abort_flag, status, kStatusTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int kk = g * 2 + h;  // k16 step within the stage
                        const uint64_t ad = umma_desc_k_sw128(base + L.a_off + ai * kCols * 128 + kk * 32);
                        const uint64_t bd = umma_desc_k_sw128(base + L.bx_off + st * 2048 + kk * 32);
                        umma_f16_ss(tmem_base + static_cast<uint32_t>(slot * 16), ad, bd, idesc, h);
                    }
                    umma_commit(d_full(slot));
                }
                umma_commit(a_empty(ai));
            }
        }
    } else if (warp >= kDqWarp0 && warp < kDqWarp0 + kDqWarps) {
        // --------------------------------------------------------- dequant --
        const int dt = tid - kDqWarp0 * 32;  // 0..127, two (column, half) units each
        for (int st = 0; st < NST; ++st) {
            const int ai = st % kAStages;
            if (!mbar_wait(raw_full(st), 0u, abort_flag, status, kStatusTimeoutDequant)) break;
            if (st >= kAStages &&
                !mbar_wait(a_empty(ai), ((st / kAStages) - 1) & 1u, abort_flag, status, kStatusTimeoutDequant))
                break;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int u = dt + i * 128;
                const int nl = u >> 1, hh = u & 1;
                const uint4 q = *reinterpret_cast<const uint4*>(smem + L.raw_off + st * kCols * 32 + nl * 32 + hh * 16);
                uint8_t* arow = smem + L.a_off + ai * kCols * 128 + nl * 128;
                const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int chunk = (hh * 4 + j) ^ (nl & 7);
                    *reinterpret_cast<uint4*>(arow + chunk * 16) = unpack_word_f16(words[j]);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(a_full(ai));
        }
    } else if (warp >= kScWarp0) {
        // ----------------------------------------------------------- scale --
        float acc[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) acc[m] = 0.0f;
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
        for (int gi = 0; gi < GS; ++gi) {
            const int slot = gi % kSlots;
            if (!mbar_wait(d_full(slot), (gi / kSlots) & 1u, abort_flag, status, kStatusTimeoutEpilogue)) break;
            tc_fence_after_sync();
            uint32_t r[16];
            tmem_ld16(lane_base + static_cast<uint32_t>(slot * 16), r);
            tmem_ld_wait();
            // select the group's scale without dynamic register indexing
            float s = 0.0f;
#pragma unroll
            for (int g = 0; g < kMaxGroups; ++g) s = (g == gi) ? sc[g] : s;
#pragma unroll
            for (int m = 0; m < 8; ++m)
                acc[m] = fmaf(s, __uint_as_float(r[m]) + __uint_as_float(r[8 + m]), acc[m]);
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(d_empty(slot));
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) part[col * 8 + m] = acc[m] * exp2i(-row_exponent(__int_as_float(row_max[m])));
    }

    // ------------------------------------- cross-slice sum, LoRA, store --
    tc_fence_before_sync();
    cluster.sync();
    if (*abort_flag == 0) {
        const int per = kCols / S;  // columns reduced by this CTA
        for (int idx = tid; idx < per * M; idx += kThreads) {
            const int cl = crank * per + idx / M, m = idx % M;
            const int n = n0 + cl;
            if (n >= N) continue;
            float sum = 0.0f;
            for (int r = 0; r < S; ++r) sum += cluster.map_shared_rank(part, r)[cl * 8 + m];
            if (lora_t != nullptr) {
                float d = 0.0f;
                for (int j = 0; j < rank; ++j) d = fmaf(lora_t[m * rank + j], lora_b[static_cast<size_t>(j) * N + n], d);
                sum = fmaf(lora_scale, d, sum);
            }
            y[static_cast<size_t>(m) * N + n] = sum;
        }
    } else if (warp == 0 && lane == 0) {
        for (int st = 0; st < NST; ++st) mbar_drain(raw_full(st), 0u);  // copies in flight land first
    }
    cluster.sync();  // partials stay alive until every peer has read them
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc(tmem_base, kSlots * 16);
    }
}

}  // namespace

bool decode_supported(int M, int K, int S) {
    if (M < 1 || M > 8 || S < 1 || S > 8 || K % 32) return false;
    const int G = K / 32;
    if (G % S) return false;
    const int GS = G / S;
    return GS % 2 == 0 && GS >= 2 && GS <= kMaxGroups;
}

size_t decode_smem_bytes(int K, int S) { return static_cast<size_t>(decode_layout(K, S).bytes) + 1024; }

int decode_columns_per_cluster() { return kCols; }

int launch_decode(const GemvArgs& a, cudaStream_t stream) {
    const int S = a.cluster_k;
    const size_t smem = decode_smem_bytes(a.K, S);
    cudaError_t e =
        cudaFuncSetAttribute(q4_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
    const int blocks = (a.N + kCols - 1) / kCols;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(S * blocks), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
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
    e = cudaLaunchKernelEx(&cfg, q4_decode_kernel, a.tmap_w, a.x, a.scales, a.y, a.M, a.N, a.K, a.lora_t, a.lora_b,
                           a.rank, a.lora_scale, a.status);
    return static_cast<int>(e);
}

}  // namespace q4
