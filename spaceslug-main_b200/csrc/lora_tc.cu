// LoRA adapter gradients on the tcgen05 tensor cores (fp32 operands,
// fp32-level accuracy), the large-M form of the backward in lora_train.cu:
//
//   T  = X A        [M x r]        G  = dY B^T      [M x r]
//   dB = s T^T dY   [r x N]        dA = s X^T G     [K x r]
//
// (the reference's lora_gradients, vulkan-runtime/src/api/lora_gradients_api.h:4-6,
// dA = X^T dY B^T and dB = (X A)^T dY, here with s = alpha / rank and any rank <= 64).
//
// Each of the four contractions has the shape
//   D[R x r] = sum over l < L of  Aop[row][l] * Bop[j][l]
// with one wide fp32 operand Aop (X or dY, streamed from HBM once per
// contraction) and one narrow operand Bop of r rows (A^T, B, T^T or G^T).
// lora_tc_kernel<RP, MN> runs all four:
//
//  - Aop is TMA-loaded in tiles of 128 rows x 32 l straight from X or dY,
//    either with the rows of D as the source's rows (T and G: l contiguous)
//    or with the rows of D contiguous in the source (dB reads dY^T and dA
//    reads X^T: four 32 x 32 boxes per tile).
//  - Four split warps turn each loaded tile into TF32 hi (rounded to nearest)
//    and lo = x - hi (exact in fp32) in shared memory, K-major and
//    128-byte-swizzled for the MMA: in place for the first kind; for the
//    second, through 4 x 4 register transposes from the loaded tile into two
//    further tiles (the MMA's MN-major TF32 operand form needs another
//    swizzle layout, so the transpose happens here).  Neither the split nor a
//    transpose ever passes through HBM.
//  - Bop is prepared once per contraction as stacked planes [2RP][L]: rows
//    0..RP-1 its TF32 hi parts, rows RP..2RP-1 its lo parts, rows >= r zero.
//    Two MMAs per 8 l, Aop_hi x [B_hi; B_lo] and Aop_lo x [B_hi; B_lo]
//    (kind::tf32, M = 128, N = 2RP, K = 8), form all four hi / lo cross
//    products; D[:, j] + D[:, RP + j] is the product to fp32 accuracy.
//  - The accumulator is double-buffered in tensor memory and restarted every
//    32 l: four epilogue warps add each finished chunk to fp32 sums in
//    registers with round-to-nearest (the tensor cores accumulate with
//    truncation, a bias that grows with the contraction length).  Two warps
//    issue the MMAs, of even and of odd stages.
//  - Work units are (128-row tile, range of l) pairs.  A persistent grid of
//    one CTA per SM walks them; each unit writes its partial D to
//    partial[split][row][RP], and lora_tc_finalize_kernel sums the splits in
//    a fixed order (deterministic) and writes the result in the layout the
//    next step reads.
// Every wait is bounded (status word + abort flag).
#include <cuda.h>
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>

#include "common.cuh"
#include "q4_kernels.h"

namespace q4 {

namespace {

constexpr int kLtRows = 128;      // rows of D per unit (the MMA's M)
constexpr int kLtL = 32;          // contraction elements per stage: one 128-byte fp32 row
// Warps: 0 TMA, 1 and 10 MMA, 4-7 epilogue, split: 2-3 and 8-9, plus 11-14
// for the transposing split (MN), which costs about twice as much per stage.
template <bool MN>
__host__ __device__ constexpr int lt_split_warps() { return MN ? 8 : 4; }
template <bool MN>
__host__ __device__ constexpr int lt_threads() { return MN ? 480 : 352; }
__device__ __forceinline__ int lt_split_index(int warp) {  // split warp -> 0..7, else -1
    return (warp == 2 || warp == 3) ? warp - 2 : (warp == 8 || warp == 9) ? warp - 6 : warp >= 11 ? warp - 7 : -1;
}
constexpr int kLtATile = kLtRows * kLtL * 4;  // 16 KB

template <int RP, bool MN>
struct LtCfg {
    static constexpr int kBTile = 2 * RP * kLtL * 4;  // stacked hi / lo rows of Bop
    static constexpr int kBTileAligned = (kBTile + 1023) / 1024 * 1024;
    // stage: [loaded Aop (MN only)] [Aop hi] [Aop lo] [Bop]; without MN the hi tile is the loaded one
    static constexpr int kHi = MN ? kLtATile : 0;
    static constexpr int kLo = kHi + kLtATile;
    static constexpr int kB = kLo + kLtATile;
    static constexpr int kStageBytes = kB + kBTileAligned;
    static constexpr int kBudget = 222 * 1024;
    static constexpr int kStages = kBudget / kStageBytes > 8 ? 8 : kBudget / kStageBytes;
    static constexpr int kTmemCols = 4 * RP < 32 ? 32 : 4 * RP;  // two chunk buffers of 2RP columns
    static_assert(kStages > 2, "the epilogue waits on the stages' MMA commits: it must not fall a phase behind");
    static constexpr int kBarOff = kStages * kStageBytes;
    // full[S], split[S], empty[S], chunk_empty[2]; then abort flag, TMEM address
    static constexpr int kNumBars = 3 * kStages + 2;
    static constexpr int kSmem = kBarOff + kNumBars * 8 + 16;
    static constexpr int kSmemAlloc = kSmem + 1024;  // slack to align the window to 1024
};

// Unit u of a pass: 128-row tile `tile`, split z, stages [s0, s1) of the NS
// 32-l stages (splits <= NS, so every unit has at least one stage).
__device__ __forceinline__ void lt_unit(int u, int tiles, int splits, int NS, int& tile, int& z, int& s0, int& s1) {
    tile = u % tiles;
    z = u / tiles;
    s0 = static_cast<int>(static_cast<long long>(z) * NS / splits);
    s1 = static_cast<int>(static_cast<long long>(z + 1) * NS / splits);
}

// Stages this CTA processes in all (every role walks the same sequence).
__device__ __forceinline__ int lt_total_stages(int tiles, int splits, int NS) {
    int n = 0;
    for (int u = blockIdx.x; u < tiles * splits; u += gridDim.x) {
        int tile, z, s0, s1;
        lt_unit(u, tiles, splits, NS, tile, z, s0, s1);
        n += s1 - s0;
    }
    return n;
}

template <int RP, bool MN>
__global__ void __launch_bounds__(lt_threads<MN>(), 1)
    lora_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   float* __restrict__ partial, int R, int L, int splits, int* __restrict__ status) {
    using C = LtCfg<RP, MN>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // 128B-swizzled tiles need a 1024-aligned window
    uint8_t* smem = smem_raw + (base - raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tiles = (R + kLtRows - 1) / kLtRows;
    const int units = tiles * splits;
    const int NS = (L + kLtL - 1) / kLtL;

    const uint32_t bar = base + C::kBarOff;
    auto full = [&](int s) { return bar + 8u * s; };
    auto split = [&](int s) { return bar + 8u * (C::kStages + s); };
    auto empty = [&](int s) { return bar + 8u * (2 * C::kStages + s); };
    auto chunk_empty = [&](int b) { return bar + 8u * (3 * C::kStages + b); };
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kBarOff + C::kNumBars * 8);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kBarOff + C::kNumBars * 8 + 8);

    if (tid == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(full(s), 1);
            mbar_init(split(s), lt_split_warps<MN>());
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) mbar_init(chunk_empty(b), 4);  // one arrival per epilogue warp
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    pdl_launch_dependents();
    pdl_wait();  // Bop (and Aop) may be written by the previous launch

    if (warp == 0) {
        if (lane == 0) {
            // --------------------------------------------------- producer --
            tma_prefetch_desc(&tm_a);
            tma_prefetch_desc(&tm_b);
            int q = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                int tile, z, s0, s1;
                lt_unit(u, tiles, splits, NS, tile, z, s0, s1);
                const int row0 = tile * kLtRows;
                for (int st = s0; st < s1; ++st, ++q) {
                    const int s = q % C::kStages;
                    if (q >= C::kStages &&
                        !mbar_wait(empty(s), ((q / C::kStages) - 1) & 1u, abort_flag, status, kStatusTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    const uint32_t a = base + s * C::kStageBytes;
                    mbar_arrive_expect_tx(full(s), static_cast<uint32_t>(kLtATile + C::kBTile));
                    const int l0 = st * kLtL;
                    if constexpr (MN) {
                        // four boxes of 32 rows of D x 32 l (l = the box's row), 4 KB apart
#pragma unroll
                        for (int b = 0; b < 4; ++b) tma_load_2d(a + b * 4096, &tm_a, full(s), row0 + 32 * b, l0);
                    } else {
                        tma_load_2d(a, &tm_a, full(s), l0, row0);
                    }
                    tma_load_2d(a + C::kB, &tm_b, full(s), l0, 0);
                }
            }
            if (*abort_flag)  // let copies in flight land before the CTA exits
                for (int j = q > C::kStages ? q - C::kStages : 0; j < q; ++j)
                    mbar_drain(full(j % C::kStages), (j / C::kStages) & 1u);
        }
        __syncwarp();
    } else if (warp == 1 || warp == 10) {
        if (lane == 0) {
            // -------------------------------------------------------- MMA --
            // Warp 1 issues the even stages into chunk buffer 0, warp 10 the
            // odd ones into buffer 1: one thread alone cannot issue the small
            // MMAs of a 16-KB stage as fast as HBM delivers them.  One commit
            // per stage tells both the producer (the stage may be refilled) and
            // the epilogue (the chunk's sums are complete).
            const int par = warp == 1 ? 0 : 1;
            constexpr uint32_t idesc = umma_idesc_tf32(kLtRows, 2 * RP);
            const int total = lt_total_stages(tiles, splits, NS);
            const uint32_t dacc = tmem + static_cast<uint32_t>(par * 2 * RP);
            int last = -1;
            for (int q = par; q < total; q += 2) {
                const int s = q % C::kStages;
                if (q >= 2 && !mbar_wait(chunk_empty(par), ((q >> 1) - 1) & 1u, abort_flag, status, kStatusTimeoutMma))
                    break;
                if (!mbar_wait(split(s), (q / C::kStages) & 1u, abort_flag, status, kStatusTimeoutMma)) break;
                tc_fence_after_sync();
                const uint32_t st_base = base + s * C::kStageBytes;
                const uint32_t a_hi = st_base + C::kHi, a_lo = st_base + C::kLo, bt = st_base + C::kB;
#pragma unroll
                for (int kk = 0; kk < kLtL / 8; ++kk) {  // 8 tf32 = 32 bytes of each 128-byte row
                    const uint64_t bd = umma_desc_k_sw128(bt + kk * 32);
                    umma_tf32_ss(dacc, umma_desc_k_sw128(a_hi + kk * 32), bd, idesc, kk > 0 ? 1u : 0u);
                    umma_tf32_ss(dacc, umma_desc_k_sw128(a_lo + kk * 32), bd, idesc, 1u);
                }
                umma_commit(empty(s));
                last = q;
            }
            if (*abort_flag && last >= 0)  // issued MMAs finish before tensor memory is freed
                mbar_drain(empty(last % C::kStages), (last / C::kStages) & 1u);
        }
        __syncwarp();
    } else if (warp >= 4 && warp < 8) {
        // -------------------------------------------------------- epilogue --
        // Warp w reads TMEM lane quarter w % 4: thread t <-> row 32 (w % 4) + t of the tile.
        const int quarter = warp & 3;
        const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        int q = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
            int tile, z, s0, s1;
            lt_unit(u, tiles, splits, NS, tile, z, s0, s1);
            float total[RP];
#pragma unroll
            for (int j = 0; j < RP; ++j) total[j] = 0.0f;
            for (int st = s0; st < s1; ++st, ++q) {
                const int b = q & 1;
                if (!mbar_wait_warp(empty(q % C::kStages), (q / C::kStages) & 1u, abort_flag, status,
                                    kStatusTimeoutEpilogue)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t col = t_lane + static_cast<uint32_t>(b * 2 * RP);
                if constexpr (RP == 8) {
                    uint32_t v[16];
                    tmem_ld16(col, v);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 8; ++j) total[j] += __uint_as_float(v[j]) + __uint_as_float(v[8 + j]);
                } else {
#pragma unroll
                    for (int cb = 0; cb < RP; cb += 16) {
                        uint32_t h[16], l[16];
                        tmem_ld16(col + cb, h);
                        tmem_ld16(col + RP + cb, l);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 16; ++j) total[cb + j] += __uint_as_float(h[j]) + __uint_as_float(l[j]);
                    }
                }
                tc_fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(chunk_empty(b));  // buffer b may take chunk q + 2
            }
            if (!ok) break;
            const int row = tile * kLtRows + quarter * 32 + lane;
            if (row < R) {
                float4* dst = reinterpret_cast<float4*>(partial + (static_cast<size_t>(z) * R + row) * RP);
#pragma unroll
                for (int j = 0; j < RP; j += 4)
                    dst[j / 4] = make_float4(total[j], total[j + 1], total[j + 2], total[j + 3]);
            }
        }
    } else if (lt_split_index(warp) >= 0) {
        // ----------------------------------------------------------- split --
        // Warps 2, 3, 8, 9 write each stage's Aop as K-major TF32 hi and lo
        // tiles (rows of D at 128 B, 16-byte chunk c of row m at c ^ (m & 7)).
        constexpr int kSplitThreads = lt_split_warps<MN>() * 32;
        const int ct = lt_split_index(warp) * 32 + lane;  // 0 .. kSplitThreads - 1
        int q = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
            int tile, z, s0, s1;
            lt_unit(u, tiles, splits, NS, tile, z, s0, s1);
            for (int st = s0; st < s1; ++st, ++q) {
                const int s = q % C::kStages;
                if (!mbar_wait_warp(full(s), (q / C::kStages) & 1u, abort_flag, status, kStatusTimeoutDequant)) {
                    ok = false;
                    break;
                }
                uint8_t* stage = smem + s * C::kStageBytes;
                if constexpr (MN) {
                    // Loaded: box b (rows 32b..32b+31 of D) at 4 KB b, l at 128 B l, chunk (row / 4 % 8) ^ (l & 7).
                    // Each thread moves two 4 x 4 blocks (rows 4c.., l 4d..): four 16-byte reads, a register
                    // transpose, four 16-byte writes per plane.  A phase of 8 lanes spans 4 c and 2 d, so its
                    // reads hit 8 distinct chunk positions and its writes 4.
#pragma unroll
                    for (int rep = 0; rep < 256 / kSplitThreads; ++rep) {
                        const int k = ct + kSplitThreads * rep, p = k >> 3, qq = k & 7;
                        const int c = (qq & 3) + 4 * (p & 7);     // rows 4c..4c+3 of D
                        const int d = (qq >> 2) + 2 * (p >> 3);   // l = 4d..4d+3
                        float4 v[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int l = 4 * d + i;
                            v[i] = *reinterpret_cast<const float4*>(stage + 4096 * (c >> 3) + 128 * l +
                                                                    (((c & 7) ^ (l & 7)) << 4));
                        }
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj) {
                            const int row = 4 * c + jj;
                            const float4 x = jj == 0   ? make_float4(v[0].x, v[1].x, v[2].x, v[3].x)
                                             : jj == 1 ? make_float4(v[0].y, v[1].y, v[2].y, v[3].y)
                                             : jj == 2 ? make_float4(v[0].z, v[1].z, v[2].z, v[3].z)
                                                       : make_float4(v[0].w, v[1].w, v[2].w, v[3].w);
                            const float4 h = make_float4(to_tf32(x.x), to_tf32(x.y), to_tf32(x.z), to_tf32(x.w));
                            const int off = 128 * row + ((d ^ (row & 7)) << 4);
                            *reinterpret_cast<float4*>(stage + C::kHi + off) = h;
                            *reinterpret_cast<float4*>(stage + C::kLo + off) =
                                make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
                        }
                    }
                } else {
                    // Loaded K-major already: hi in place, lo at the same offsets (so the same swizzle).
                    float4* hi = reinterpret_cast<float4*>(stage + C::kHi);
                    float4* lo = reinterpret_cast<float4*>(stage + C::kLo);
                    constexpr int kPer = kLtATile / 16 / kSplitThreads;  // 8 float4 per thread
                    float4 v[kPer];
#pragma unroll
                    for (int i = 0; i < kPer; ++i) v[i] = hi[ct + kSplitThreads * i];
#pragma unroll
                    for (int i = 0; i < kPer; ++i) {
                        const float4 h =
                            make_float4(to_tf32(v[i].x), to_tf32(v[i].y), to_tf32(v[i].z), to_tf32(v[i].w));
                        hi[ct + kSplitThreads * i] = h;
                        lo[ct + kSplitThreads * i] = make_float4(v[i].x - h.x, v[i].y - h.y, v[i].z - h.z, v[i].w - h.w);
                    }
                }
                fence_proxy_async_smem();  // the MMAs (async proxy) read what these threads wrote
                __syncwarp();
                if (lane == 0) mbar_arrive(split(s));
            }
        }
    }
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

// v[row][j] = sum over z < splits of src[z][row][j] in order z = 0, 1, ...
// (row pitch `pitch`; columns j >= r read as zero), then
//   mode 0: stacked TF32 planes of v^T: out[j][row] = hi(v), out[RP + j][row] = lo(v), rows r..RP-1 zero;
//   mode 1: out[j][row] = s v (r rows, row pitch ld);
//   mode 2: out[row][j] = s v (row pitch ld).
// One block per 32 rows, transposed through shared memory so both sides stay coalesced.
__global__ void __launch_bounds__(256) lora_tc_finalize_kernel(const float* __restrict__ src, int splits, int R,
                                                               int pitch, int r, int RP, float s, int mode,
                                                               float* __restrict__ out, long long ld) {
    __shared__ float tile[32][65];
    pdl_launch_dependents();
    pdl_wait();
    const int r0 = blockIdx.x * 32;
    for (int i = threadIdx.x; i < 32 * RP; i += 256) {
        const int rr = i / RP, j = i % RP, row = r0 + rr;
        float v = 0.0f;
        if (row < R && j < r)
            for (int z = 0; z < splits; ++z) v += src[(static_cast<size_t>(z) * R + row) * pitch + j];
        tile[rr][j] = v;
    }
    __syncthreads();
    if (mode == 0) {
        for (int i = threadIdx.x; i < RP * 32; i += 256) {
            const int j = i / 32, rr = i % 32, row = r0 + rr;
            if (row >= R) continue;
            const float v = tile[rr][j], h = to_tf32(v);
            out[static_cast<size_t>(j) * ld + row] = h;
            out[static_cast<size_t>(RP + j) * ld + row] = v - h;
        }
    } else if (mode == 1) {
        for (int i = threadIdx.x; i < r * 32; i += 256) {
            const int j = i / 32, rr = i % 32, row = r0 + rr;
            if (row < R) out[static_cast<size_t>(j) * ld + row] = s * tile[rr][j];
        }
    } else {
        for (int i = threadIdx.x; i < 32 * r; i += 256) {
            const int rr = i / r, j = i % r, row = r0 + rr;
            if (row < R) out[static_cast<size_t>(row) * ld + j] = s * tile[rr][j];
        }
    }
}

// Stacked TF32 planes of a row-major [r][C] matrix, same orientation:
// plane[j][c] = hi(src[j][c]), plane[RP + j][c] = lo, rows r..RP-1 zero.
__global__ void __launch_bounds__(256) lora_tc_stack_kernel(const float* __restrict__ src, int r, int C,
                                                            long long ld_src, int RP, float* __restrict__ plane,
                                                            long long ld) {
    pdl_launch_dependents();
    pdl_wait();
    const long long total = static_cast<long long>(RP) * C;
    for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += static_cast<long long>(gridDim.x) * 256) {
        const int j = static_cast<int>(i / C);
        const long long c = i - static_cast<long long>(j) * C;
        const float v = j < r ? src[static_cast<long long>(j) * ld_src + c] : 0.0f;
        const float h = to_tf32(v);
        plane[static_cast<long long>(j) * ld + c] = h;
        plane[static_cast<long long>(RP + j) * ld + c] = v - h;
    }
}

template <typename Kern, typename... Args>
int launch_pdl(Kern kern, dim3 grid, dim3 block, int smem, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return static_cast<int>(cudaLaunchKernelEx(&cfg, kern, args...));
}

template <int RP, bool MN>
int launch_pass_rp(const LoraTcPass& p, cudaStream_t stream) {
    using C = LtCfg<RP, MN>;
    auto kern = lora_tc_kernel<RP, MN>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemAlloc);
    if (e != cudaSuccess) return static_cast<int>(e);
    const long long units = static_cast<long long>((p.R + kLtRows - 1) / kLtRows) * p.splits;
    const int grid = static_cast<int>(units < p.sm_count ? units : p.sm_count);
    return launch_pdl(kern, dim3(static_cast<unsigned>(grid)), dim3(lt_threads<MN>()), C::kSmemAlloc, stream, p.tm_a,
                      p.tm_b, p.partial, p.R, p.L, p.splits, p.status);
}

}  // namespace

int lora_tc_rp(int rank) {
    if (rank <= 8) return 8;
    if (rank <= 16) return 16;
    if (rank <= 32) return 32;
    return 64;
}

int lora_tc_splits(int R, int L, int sm_count) {
    const int tiles = (R + kLtRows - 1) / kLtRows, NS = (L + kLtL - 1) / kLtL;
    const int smax = NS < 32 ? NS : 32;
    int best = 1;
    long long best_t = LLONG_MAX;
    for (int S = 1; S <= smax; ++S) {
        const long long units = static_cast<long long>(tiles) * S;
        const long long waves = (units + sm_count - 1) / sm_count;
        // per-CTA stages, plus about two stages of fill and store per unit
        const long long t = waves * ((NS + S - 1) / S + 2);
        if (t < best_t) {
            best_t = t;
            best = S;
        }
    }
    return best;
}

int launch_lora_tc_pass(const LoraTcPass& p, cudaStream_t stream) {
    if (p.R < 1 || p.L < 1 || p.splits < 1 || p.splits > (p.L + kLtL - 1) / kLtL || p.sm_count < 1)
        return static_cast<int>(cudaErrorInvalidValue);
    const bool mn = p.mn_major != 0;
    switch (p.rp) {
        case 8: return mn ? launch_pass_rp<8, true>(p, stream) : launch_pass_rp<8, false>(p, stream);
        case 16: return mn ? launch_pass_rp<16, true>(p, stream) : launch_pass_rp<16, false>(p, stream);
        case 32: return mn ? launch_pass_rp<32, true>(p, stream) : launch_pass_rp<32, false>(p, stream);
        case 64: return mn ? launch_pass_rp<64, true>(p, stream) : launch_pass_rp<64, false>(p, stream);
        default: return static_cast<int>(cudaErrorInvalidValue);
    }
}

int launch_lora_tc_finalize(const float* src, int splits, int R, int pitch, int r, int rp, float s, int mode,
                            float* out, long long ld, cudaStream_t stream) {
    if (R < 1 || splits < 1 || r < 1 || r > rp || rp > 64 || mode < 0 || mode > 2)
        return static_cast<int>(cudaErrorInvalidValue);
    return launch_pdl(lora_tc_finalize_kernel, dim3(static_cast<unsigned>((R + 31) / 32)), dim3(256), 0, stream, src,
                      splits, R, pitch, r, rp, s, mode, out, ld);
}

int launch_lora_tc_stack(const float* src, int r, int C, long long ld_src, int rp, float* plane, long long ld,
                         cudaStream_t stream) {
    if (r < 1 || r > rp || C < 1) return static_cast<int>(cudaErrorInvalidValue);
    long long blocks = (static_cast<long long>(rp) * C + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    return launch_pdl(lora_tc_stack_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, src, r, C,
                      ld_src, rp, plane, ld);
}

}  // namespace q4
