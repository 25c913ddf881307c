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
//    either with the rows of D as the source's rows (T and G: l contiguous,
//    one 128-byte-swizzled box) or with the rows of D contiguous in the
//    source (dB reads dY^T and dA reads X^T: one unswizzled box of 32 l x 128
//    rows, 512 contiguous bytes per l).
//  - Four split warps, one per tensor-memory lane quarter, give each row of
//    the tile to one thread: it reads the row's 32 values from shared memory
//    (a 128-byte swizzled row, or one 4-byte column of the l-major box:
//    conflict-free either way), forms TF32 hi (rounded to nearest) and
//    lo = x - hi (exact in fp32) and stores both into tensor memory, where
//    the MMAs read them as the A operand (row = lane).  So the transpose of
//    the second kind costs nothing, and shared memory carries each tile once
//    in (TMA) and once out (the split) instead of also holding the hi / lo
//    tiles for the MMA to read.
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
// Warps: 0 TMA, 1 and 10 MMA, 2-3 and 8-9 split, 4-7 epilogue.
constexpr int kLtSplitWarps = 4;
constexpr int kLtThreads = 352;
__device__ __forceinline__ int lt_split_index(int warp) {  // split warp -> 0..3, else -1
    return (warp == 2 || warp == 3) ? warp - 2 : (warp == 8 || warp == 9) ? warp - 6 : -1;
}
constexpr int kLtATile = kLtRows * kLtL * 4;  // 16 KB
constexpr int kLtTmemCols = 512;              // the whole of tensor memory (one CTA per SM)

template <int RP, bool MN>
struct LtCfg {
    static constexpr int kBTile = 2 * RP * kLtL * 4;  // stacked hi / lo rows of Bop
    static constexpr int kBTileAligned = (kBTile + 1023) / 1024 * 1024;
    // shared-memory stage: [Aop as loaded] [Bop]
    static constexpr int kB = kLtATile;
    static constexpr int kStageBytes = kB + kBTileAligned;
    static constexpr int kBudget = 222 * 1024;
    static constexpr int kSmemStages = kBudget / kStageBytes;
    // tensor memory: columns [0, 4RP) two accumulator chunk buffers of 2RP columns;
    // from kACol on, per stage 64 columns: 32 of Aop hi (one l per column), 32 of Aop lo
    static constexpr int kACol = 4 * RP < 64 ? 64 : 4 * RP;
    static constexpr int kTmemStages = (kLtTmemCols - kACol) / 64;
    static constexpr int kStages0 = kSmemStages < kTmemStages ? kSmemStages : kTmemStages;
    static constexpr int kStages = kStages0 > 8 ? 8 : kStages0;
    static_assert(kStages > 2, "the epilogue waits on the stages' MMA commits: it must not fall a phase behind");
    static constexpr int kBarOff = kStages * kStageBytes;
    // full[S], split[S], empty[S], chunk_empty[2]; then abort flag, TMEM address
    static constexpr int kNumBars = 3 * kStages + 2;
    static constexpr int kSmem = kBarOff + kNumBars * 8 + 16;
    static constexpr int kSmemAlloc = kSmem + 1024;  // slack to align the window to 1024
};

// Unit u of a launch: problem pi, 128-row tile, split z, stages [s0, s1) of
// the problem's NS 32-l stages (splits <= NS, so every unit has at least one
// stage).  The first problem's units come first.
struct LtUnit {
    int pi, tile, z, s0, s1;
};
__device__ __forceinline__ int lt_units(const LoraTcProblem& q) { return (q.R + kLtRows - 1) / kLtRows * q.splits; }
__device__ __forceinline__ LtUnit lt_unit(const LoraTcPass& P, int u) {
    LtUnit w;
    const int u0 = lt_units(P.prob[0]);
    w.pi = (P.count > 1 && u >= u0) ? 1 : 0;
    const LoraTcProblem& q = P.prob[w.pi];
    const int lu = w.pi ? u - u0 : u;
    const int tiles = (q.R + kLtRows - 1) / kLtRows, NS = (q.L + kLtL - 1) / kLtL;
    w.tile = lu % tiles;
    w.z = lu / tiles;
    w.s0 = static_cast<int>(static_cast<long long>(w.z) * NS / q.splits);
    w.s1 = static_cast<int>(static_cast<long long>(w.z + 1) * NS / q.splits);
    return w;
}

template <int RP, bool MN>
__global__ void __launch_bounds__(kLtThreads, 1)
    lora_tc_kernel(const __grid_constant__ LoraTcPass P) {
    using C = LtCfg<RP, MN>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // 128B-swizzled tiles need a 1024-aligned window
    uint8_t* smem = smem_raw + (base - raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int units = lt_units(P.prob[0]) + (P.count > 1 ? lt_units(P.prob[1]) : 0);
    int* status = P.status;

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
            mbar_init(split(s), kLtSplitWarps);
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) mbar_init(chunk_empty(b), 4);  // one arrival per epilogue warp
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), kLtTmemCols);
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
            for (int i = 0; i < P.count; ++i) {
                tma_prefetch_desc(&P.prob[i].tm_a);
                tma_prefetch_desc(&P.prob[i].tm_b);
            }
            int q = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                const LtUnit w = lt_unit(P, u);
                const CUtensorMap* tm_a = &P.prob[w.pi].tm_a;
                const CUtensorMap* tm_b = &P.prob[w.pi].tm_b;
                const int row0 = w.tile * kLtRows;
                for (int st = w.s0; st < w.s1; ++st, ++q) {
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
                        tma_load_2d(a, tm_a, full(s), row0, l0);  // [32 l][128 rows of D], 512-byte rows
                    } else {
                        tma_load_2d(a, tm_a, full(s), l0, row0);  // [128 rows][32 l], 128-byte swizzled rows
                    }
                    tma_load_2d(a + C::kB, tm_b, full(s), l0, 0);
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
            int total = 0;
            for (int u = blockIdx.x; u < units; u += gridDim.x) {
                const LtUnit w = lt_unit(P, u);
                total += w.s1 - w.s0;
            }
            const uint32_t dacc = tmem + static_cast<uint32_t>(par * 2 * RP);
            int last = -1;
            for (int q = par; q < total; q += 2) {
                const int s = q % C::kStages;
                if (q >= 2 && !mbar_wait(chunk_empty(par), ((q >> 1) - 1) & 1u, abort_flag, status, kStatusTimeoutMma))
                    break;
                if (!mbar_wait(split(s), (q / C::kStages) & 1u, abort_flag, status, kStatusTimeoutMma)) break;
                tc_fence_after_sync();
                const uint32_t bt = base + s * C::kStageBytes + C::kB;
                const uint32_t a_hi = tmem + static_cast<uint32_t>(C::kACol + 64 * s), a_lo = a_hi + 32;
#pragma unroll
                for (int kk = 0; kk < kLtL / 8; ++kk) {  // K = 8: 8 columns of A, 32 bytes of each B row
                    const uint64_t bd = umma_desc_k_sw128(bt + kk * 32);
                    umma_tf32_ts(dacc, a_hi + 8 * kk, bd, idesc, kk > 0 ? 1u : 0u);
                    umma_tf32_ts(dacc, a_lo + 8 * kk, bd, idesc, 1u);
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
            const LtUnit w = lt_unit(P, u);
            const LoraTcProblem& pb = P.prob[w.pi];
            float total[RP];
#pragma unroll
            for (int j = 0; j < RP; ++j) total[j] = 0.0f;
            for (int st = w.s0; st < w.s1; ++st, ++q) {
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
            const int row = w.tile * kLtRows + quarter * 32 + lane;
            if (row < pb.R) {
                float4* dst = reinterpret_cast<float4*>(pb.partial + (static_cast<size_t>(w.z) * pb.R + row) * RP);
#pragma unroll
                for (int j = 0; j < RP; j += 4)
                    dst[j / 4] = make_float4(total[j], total[j + 1], total[j + 2], total[j + 3]);
            }
        }
    } else if (lt_split_index(warp) >= 0) {
        // ----------------------------------------------------------- split --
        // Warps 2, 3, 8, 9 (lane quarters 2, 3, 0, 1): thread <-> row 32 (warp % 4) + lane
        // of the tile, whose hi and lo parts go to its tensor-memory lane.
        const int quarter = warp & 3, row = quarter * 32 + lane;
        const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        int q = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
            const LtUnit w = lt_unit(P, u);
            for (int st = w.s0; st < w.s1; ++st, ++q) {
                const int s = q % C::kStages;
                if (!mbar_wait_warp(full(s), (q / C::kStages) & 1u, abort_flag, status, kStatusTimeoutDequant)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();  // the MMAs that last read this stage's tensor memory have completed
                const uint8_t* stage = smem + s * C::kStageBytes;
                float v[kLtL];
                if constexpr (MN) {
                    // l at 512 B l, this row at 4 B row: a warp reads 128 consecutive bytes
                    const float* col = reinterpret_cast<const float*>(stage) + row;
#pragma unroll
                    for (int l = 0; l < kLtL; ++l) v[l] = col[kLtRows * l];
                } else {
                    // 128-byte row `row`, 16-byte chunk c at c ^ (row & 7)
#pragma unroll
                    for (int c = 0; c < kLtL / 4; ++c) {
                        const float4 f = *reinterpret_cast<const float4*>(stage + 128 * row + ((c ^ (row & 7)) << 4));
                        v[4 * c] = f.x;
                        v[4 * c + 1] = f.y;
                        v[4 * c + 2] = f.z;
                        v[4 * c + 3] = f.w;
                    }
                }
                uint32_t hi[kLtL], lo[kLtL];
#pragma unroll
                for (int l = 0; l < kLtL; ++l) {
                    const float h = to_tf32(v[l]);
                    hi[l] = __float_as_uint(h);
                    lo[l] = __float_as_uint(v[l] - h);
                }
                const uint32_t col = t_lane + static_cast<uint32_t>(C::kACol + 64 * s);
                tmem_st32(col, hi);
                tmem_st32(col + 32, lo);
                tmem_st_wait();
                tc_fence_before_sync();  // the MMAs (issued after the barrier) read what these threads stored
                __syncwarp();
                if (lane == 0) mbar_arrive(split(s));
            }
        }
    }
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc(tmem, kLtTmemCols);
    }
}

// One or two finalize steps per launch (blocks of the first come first).
struct LtFinalizeLaunch {
    LoraTcFinalize f[2];
    int count, rp, blocks0;
};

// v[row][j] = sum over z < splits of src[z][row][j] in order z = 0, 1, ...
// (row pitch `pitch`; columns j >= r read as zero), then
//   mode 0: stacked TF32 planes of v^T: out[j][row] = hi(v), out[RP + j][row] = lo(v), rows r..RP-1 zero;
//   mode 1: out[j][row] = s v (r rows, row pitch ld);
//   mode 2: out[row][j] = s v (row pitch ld);
//   mode 3: as mode 0 for v[row][j] = src[j][row] (a row-major [r][R] source with row pitch `pitch`).
// One block per 32 rows, transposed through shared memory so both sides stay coalesced.
__global__ void __launch_bounds__(256) lora_tc_finalize_kernel(const LtFinalizeLaunch F) {
    __shared__ float tile[32][65];
    pdl_launch_dependents();
    pdl_wait();
    const bool second = F.count > 1 && static_cast<int>(blockIdx.x) >= F.blocks0;
    const LoraTcFinalize& f = F.f[second ? 1 : 0];
    const int RP = F.rp, R = f.R, r = f.r, ld_src = f.pitch;
    const long long ld = f.ld;
    const int r0 = (static_cast<int>(blockIdx.x) - (second ? F.blocks0 : 0)) * 32;
    for (int i = threadIdx.x; i < 32 * RP; i += 256) {
        const int rr = i / RP, j = i % RP, row = r0 + rr;
        float v = 0.0f;
        if (row < R && j < r) {
            if (f.mode == 3) {
                v = f.src[static_cast<size_t>(j) * ld_src + row];
            } else {
                for (int z = 0; z < f.splits; ++z) v += f.src[(static_cast<size_t>(z) * R + row) * ld_src + j];
            }
        }
        tile[rr][j] = v;
    }
    __syncthreads();
    if (f.mode == 0 || f.mode == 3) {
        for (int i = threadIdx.x; i < RP * 32; i += 256) {
            const int j = i / 32, rr = i % 32, row = r0 + rr;
            if (row >= R) continue;
            const float v = tile[rr][j], h = to_tf32(v);
            f.out[static_cast<size_t>(j) * ld + row] = h;
            f.out[static_cast<size_t>(RP + j) * ld + row] = v - h;
        }
    } else if (f.mode == 1) {
        for (int i = threadIdx.x; i < r * 32; i += 256) {
            const int j = i / 32, rr = i % 32, row = r0 + rr;
            if (row < R) f.out[static_cast<size_t>(j) * ld + row] = f.s * tile[rr][j];
        }
    } else {
        for (int i = threadIdx.x; i < 32 * r; i += 256) {
            const int rr = i / r, j = i % r, row = r0 + rr;
            if (row < R) f.out[static_cast<size_t>(row) * ld + j] = f.s * tile[rr][j];
        }
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
    long long units = 0;
    for (int i = 0; i < p.count; ++i)
        units += static_cast<long long>((p.prob[i].R + kLtRows - 1) / kLtRows) * p.prob[i].splits;
    const int grid = static_cast<int>(units < p.sm_count ? units : p.sm_count);
    return launch_pdl(kern, dim3(static_cast<unsigned>(grid)), dim3(kLtThreads), C::kSmemAlloc, stream, p);
}

}  // namespace

int lora_tc_rp(int rank) {
    if (rank <= 8) return 8;
    if (rank <= 16) return 16;
    if (rank <= 32) return 32;
    return 64;
}

// Splits chosen together so that the problems' units have about the same
// number of stages (t) and the launch's units fill whole waves of the SMs:
// the cost of a candidate is waves x (longest unit + about two stages of
// fill and store).
void lora_tc_plan(int count, const int* R, const int* L, int sm_count, int* splits) {
    int tiles[2], NS[2], nsmax = 1;
    for (int i = 0; i < count; ++i) {
        tiles[i] = (R[i] + kLtRows - 1) / kLtRows;
        NS[i] = (L[i] + kLtL - 1) / kLtL;
        if (NS[i] > nsmax) nsmax = NS[i];
        splits[i] = 1;
    }
    long long best = LLONG_MAX;
    for (int t = 1; t <= nsmax; ++t) {
        int S[2];
        long long units = 0;
        int longest = 0;
        for (int i = 0; i < count; ++i) {
            S[i] = (NS[i] + t - 1) / t;
            if (S[i] > 64) S[i] = 64;
            if (S[i] > NS[i]) S[i] = NS[i];
            units += static_cast<long long>(tiles[i]) * S[i];
            const int len = (NS[i] + S[i] - 1) / S[i];
            if (len > longest) longest = len;
        }
        const long long cost = (units + sm_count - 1) / sm_count * (longest + 2);
        if (cost < best) {
            best = cost;
            for (int i = 0; i < count; ++i) splits[i] = S[i];
        }
    }
}

int launch_lora_tc_pass(const LoraTcPass& p, cudaStream_t stream) {
    if (p.count < 1 || p.count > 2 || p.sm_count < 1) return static_cast<int>(cudaErrorInvalidValue);
    for (int i = 0; i < p.count; ++i) {
        const LoraTcProblem& q = p.prob[i];
        if (q.R < 1 || q.L < 1 || q.splits < 1 || q.splits > (q.L + kLtL - 1) / kLtL || !q.partial)
            return static_cast<int>(cudaErrorInvalidValue);
    }
    const bool mn = p.mn_major != 0;
    switch (p.rp) {
        case 8: return mn ? launch_pass_rp<8, true>(p, stream) : launch_pass_rp<8, false>(p, stream);
        case 16: return mn ? launch_pass_rp<16, true>(p, stream) : launch_pass_rp<16, false>(p, stream);
        case 32: return mn ? launch_pass_rp<32, true>(p, stream) : launch_pass_rp<32, false>(p, stream);
        case 64: return mn ? launch_pass_rp<64, true>(p, stream) : launch_pass_rp<64, false>(p, stream);
        default: return static_cast<int>(cudaErrorInvalidValue);
    }
}

int launch_lora_tc_finalize(const LoraTcFinalize* f, int count, int rp, cudaStream_t stream) {
    if (count < 1 || count > 2 || rp < 8 || rp > 64) return static_cast<int>(cudaErrorInvalidValue);
    LtFinalizeLaunch F{};
    F.count = count;
    F.rp = rp;
    int blocks = 0;
    for (int i = 0; i < count; ++i) {
        const LoraTcFinalize& q = f[i];
        if (q.R < 1 || q.splits < 1 || q.r < 1 || q.r > rp || q.mode < 0 || q.mode > 3 || !q.src || !q.out)
            return static_cast<int>(cudaErrorInvalidValue);
        F.f[i] = q;
        if (i == 0) F.blocks0 = (q.R + 31) / 32;
        blocks += (q.R + 31) / 32;
    }
    return launch_pdl(lora_tc_finalize_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, F);
}

}  // namespace q4
