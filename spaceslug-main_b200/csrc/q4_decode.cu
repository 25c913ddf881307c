// Decode (M <= 8) on the tensor cores:  Y[M x N] = X . dequant(W) (+ LoRA), fp32
// accuracy.
//
// The reference has no decode path (q4gemm.comp:36-37 needs M % 64 == 0); the
// math is its dequant w = float(v) * scale (q4gemm.comp:104-122) and a dot
// product over K.  On CUDA cores that costs M/2 + ~2.5 fp32-pipe instructions
// per weight, which at M >= 4 is more than the HBM stream of one small layer
// leaves time for.  Here the weights are the MMA's A operand and the
// per-group scale is applied after the MMA, so a weight costs ~1.5
// instructions whatever M is:
//
//   * a CTA owns C <= 128 weight columns (the MMA's M rows / TMEM lanes) and a
//     K slice of <= 1024 (32 scale groups); the S slices of a column block are
//     the CTAs of one cluster.  N is split evenly over as many column blocks
//     as clusters fit on the GPU at once, so a launch is one wave;
//   * at entry one thread issues the TMA loads of the CTA's whole packed slice
//     (128-byte swizzled boxes of 256 k, so DRAM sees whole 128-byte rows; one
//     mbarrier per box) and the epilogue threads read
//     their column's scales: none of it depends on the previous launch, so it
//     happens before griddepcontrol.wait, as does the dequantisation of the
//     first A stages;
//   * 8 dequant warps write A = the int4 values v as f16 (exact) into a ring
//     of 128-byte-swizzled K-major tiles.  Within each 8-k word the k order is
//     (0,4,1,5,2,6,3,7): one LOP3 turns two nibbles into (1024 + v + 8) f16
//     pairs and one HSUB2 gives v; the B tiles use the same order, and a dot
//     product does not depend on it;
//   * B = X^T, 16 rows: x_hi (8 rows) and x_lo (8 rows) with x * 2^e = x_hi +
//     x_lo in f16 for a power-of-two e per (row, K slice), built from a TMA
//     copy of X after griddepcontrol.wait (v exact, x_hi + x_lo ~22 bits,
//     fp32 accumulation: ~2^-21 relative error per product);
//   * each 32-k scale group's two MMAs (K = 16) write their own 128 x 16 fp32
//     TMEM slot (32 slots = all 512 columns), so MMAs never wait for the
//     epilogue; four epilogue warps (thread = column) read slot g and
//     accumulate y[m] += s(n, g) * (D[m] + D[8 + m]);
//   * the cluster's K-slice partials are summed through distributed shared
//     memory in fixed rank order, the LoRA term is added and Y stored.
// Every wait is bounded (status word + abort flag); the CTA drains its copies
// and MMAs and frees its TMEM before it exits.
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

constexpr int kRows = 128;          // MMA M = TMEM lanes; rows >= C carry no column
constexpr int kStageK = 64;         // k per stage: one 128-byte f16 row per column
constexpr int kAStages = 4;         // dequantised A tiles in flight
constexpr int kMaxGroups = 32;      // 32 TMEM slots x 16 columns = 512
constexpr int kSlotCols = 16;       // N of each MMA: x_hi rows 0-7, x_lo rows 8-15
constexpr int kThreads = 448;       // 14 warps
constexpr int kDqWarp0 = 2;         // dequant warps 2..9
constexpr int kDqWarps = 8;         // two per A ring slot: slot p = stages p, p + 4, ...
constexpr int kEpWarp0 = 10;        // epilogue warps 10..13 (TMEM lane quarters 2, 3, 0, 1)
constexpr int kEpWarps = 4;
constexpr int kXBox = 256;          // X is copied as rows of 256 floats
constexpr int kRawBoxK = 256;       // k per packed-weight box: one 128-byte row per column

struct DLayout {
    int kslice, stages, groups, boxes, raw_box;
    int a_off, b_off, raw_off, x_off, part_off, bar_off, misc_off, bytes;
};

__host__ __device__ inline DLayout decode_layout(int M, int K, int S, int box_rows) {
    DLayout L;
    L.kslice = K / S;
    L.stages = L.kslice / kStageK;
    L.groups = L.kslice / 32;
    L.boxes = L.kslice / kRawBoxK;
    L.raw_box = box_rows * 128;                            // box_rows x 32 packed words, swizzled
    L.a_off = 0;                                           // kAStages x 16 KB (1024-aligned)
    L.b_off = L.a_off + kAStages * kRows * 128;            // stages x 2 KB (1024-aligned)
    L.raw_off = L.b_off + L.stages * 16 * 128;             // boxes x raw_box (1024-aligned)
    L.x_off = L.raw_off + L.boxes * L.raw_box;             // [M][kslice] fp32
    L.part_off = L.x_off + M * L.kslice * 4;               // [128][8] fp32
    L.bar_off = L.part_off + kRows * 8 * 4;
    // raw_full[boxes], a_full[4], stage_done[stages], x_full, b_ready, mma_done
    L.misc_off = L.bar_off + (L.boxes + kAStages + L.stages + 3) * 8;
    // tmem holder, abort flag, row exponents [8], row-max scratch [4 warps][8]
    L.bytes = L.misc_off + 16 + 8 * 4 + kEpWarps * 8 * 4;
    return L;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}

// Two nibbles (bits 0-3 and 16-19 of u) as the f16 pair (1024 + v + 8):
// (nibble ^ 8) = v + 8 goes under the exponent bits of 1024 (0x6400).
__device__ __forceinline__ uint32_t nibble_pair_f16(uint32_t u) {
    return ((u ^ 0x00080008u) & 0x000F000Fu) | 0x64006400u;
}

// The 8 int4 values of one packed word (k = 0..7 at bits 4k) as f16, exact,
// in the k order (0,4,1,5,2,6,3,7).
__device__ __forceinline__ uint4 unpack_word_f16_perm(uint32_t q) {
    const __half2 bias = __halves2half2(__ushort_as_half(0x6408u), __ushort_as_half(0x6408u));  // 1032
    uint32_t out[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t p = nibble_pair_f16(q >> (4 * i));  // (k = i, k = i + 4)
        __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&p), bias);
        out[i] = *reinterpret_cast<const uint32_t*>(&h);
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

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// Named barrier over the 128 epilogue threads.
__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 1)
    q4_decode_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                     const float* __restrict__ scales, float* __restrict__ y, int M, int N, int K, int G,
                     int box_rows, const float* __restrict__ lora_t, const float* __restrict__ lora_b, int rank,
                     float lora_scale, int* __restrict__ status) {
    extern __shared__ uint8_t smem_raw[];
    // 128-byte swizzled tiles need 1024-byte alignment in the shared window;
    // dynamic shared memory of a kernel without static shared memory starts
    // 1024-aligned.  Anything else is reported, not used.
    uint8_t* smem = smem_raw;
    const uint32_t base = smem_u32(smem_raw);
    if ((base & 1023u) != 0) {
        if (threadIdx.x == 0 && status) atomicCAS(status, 0, kStatusBadLaunch);
        return;
    }

    const int S = static_cast<int>(cluster_nctarank());
    const int crank = static_cast<int>(cluster_ctarank());
    const DLayout L = decode_layout(M, K, S, box_rows);
    const int blk = static_cast<int>(blockIdx.x) / S;
    const int n0 = static_cast<int>(static_cast<long long>(blk) * N / G);
    const int C = static_cast<int>(static_cast<long long>(blk + 1) * N / G) - n0;  // <= box_rows
    const int k0 = crank * L.kslice;
    const int g0 = k0 / 32;

    const uint32_t bar = base + L.bar_off;
    auto raw_full = [&](int b) { return bar + 8u * b; };
    auto a_full = [&](int i) { return bar + 8u * (L.boxes + i); };
    // one commit per stage: its A slot is free again and its two groups' TMEM
    // slots hold their results
    auto stage_done = [&](int st) { return bar + 8u * (L.boxes + kAStages + st); };
    const uint32_t x_full = bar + 8u * (L.boxes + kAStages + L.stages);
    const uint32_t b_ready = x_full + 8u;
    const uint32_t mma_done = x_full + 16u;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L.misc_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off + 4);
    int* row_exp = reinterpret_cast<int*>(smem + L.misc_off + 16);        // [8]
    float* row_max = reinterpret_cast<float*>(smem + L.misc_off + 48);   // [4 warps][8]
    float* part = reinterpret_cast<float*>(smem + L.part_off);            // [128][8]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int b = 0; b < L.boxes; ++b) mbar_init(raw_full(b), 1);
        for (int i = 0; i < kAStages; ++i) mbar_init(a_full(i), kDqWarps / kAStages);
        for (int st = 0; st < L.stages; ++st) mbar_init(stage_done(st), 1);
        mbar_init(x_full, 1);
        mbar_init(b_ready, 1);
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
        // The packed slice does not depend on the previous launch; it goes
        // out first, before the TMEM allocation and the CTA barrier.
        tma_prefetch_desc(&tmap_w);
        tma_prefetch_desc(&tmap_x);
        for (int b = 0; b < L.boxes; ++b) {
            mbar_arrive_expect_tx(raw_full(b), static_cast<uint32_t>(L.raw_box));
            tma_load_2d(base + L.raw_off + b * L.raw_box, &tmap_w, raw_full(b), (k0 + b * kRawBoxK) / 8, n0);
        }
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_holder), kMaxGroups * kSlotCols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_holder;
    // Epilogue threads: this column's scales for the slice (also independent).
    float sc[kMaxGroups];
    const int quarter = warp & 3;
    const int col = quarter * 32 + lane;  // TMEM lane = column within the block
    if (warp >= kEpWarp0) {
        const int n = n0 + col;
        const bool have = col < C && n < N;
        const float4* srow = reinterpret_cast<const float4*>(scales + static_cast<size_t>(have ? n : 0) * (K / 32) + g0);
#pragma unroll
        for (int g4 = 0; g4 < kMaxGroups / 4; ++g4) {
            const float4 v = (have && g4 * 4 < L.groups) ? __ldg(srow + g4) : make_float4(0.f, 0.f, 0.f, 0.f);
            sc[4 * g4] = v.x;
            sc[4 * g4 + 1] = v.y;
            sc[4 * g4 + 2] = v.z;
            sc[4 * g4 + 3] = v.w;
        }
    }
    // Dependents may launch now.  Only the X copy and the final Y/LoRA phase
    // wait for the previous launch; dequantisation runs ahead of it.
    pdl_launch_dependents();
    if (warp == 0 && lane == 0) {
        pdl_wait();
        mbar_arrive_expect_tx(x_full, static_cast<uint32_t>(M * L.kslice * 4));
        for (int m = 0; m < M; ++m)
            tma_load_2d(base + L.x_off + m * L.kslice * 4, &tmap_x, x_full, 0, m * (K / kXBox) + k0 / kXBox);
    }

    if (warp == 1) {
        // ------------------------------------------------------------- MMA --
        if (elect_one()) {
            const uint32_t idesc = umma_idesc_f16(0u, static_cast<uint32_t>(kRows), static_cast<uint32_t>(kSlotCols));
            bool ok = mbar_wait(b_ready, 0u, abort_flag, status, kStatusTimeoutMma);
            tc_fence_after_sync();
            for (int st = 0; st < L.stages && ok; ++st) {
                const int ai = st % kAStages;
                if (!mbar_wait(a_full(ai), (st / kAStages) & 1u, abort_flag, status, kStatusTimeoutMma)) break;
                tc_fence_after_sync();
#pragma unroll
                for (int g = 0; g < 2; ++g) {
                    const int gi = st * 2 + g;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int kk = g * 2 + h;  // k16 step within the stage
                        const uint64_t ad = umma_desc_k_sw128(base + L.a_off + ai * kRows * 128 + kk * 32);
                        const uint64_t bd = umma_desc_k_sw128(base + L.b_off + st * 16 * 128 + kk * 32);
                        umma_f16_ss(tmem_base + static_cast<uint32_t>(gi * kSlotCols), ad, bd, idesc, h);
                    }
                }
                umma_commit(stage_done(st));
            }
            umma_commit(mma_done);  // tracks every MMA issued above
        }
        __syncwarp();
    } else if (warp >= kDqWarp0 && warp < kDqWarp0 + kDqWarps) {
        // --------------------------------------------------------- dequant --
        // Warps 2p and 2p + 1 own A ring slot p and dequantise stages p, p + 4,
        // ... (four slots fill in parallel); each takes 64 of the 128 rows.
        // Lane unit v = lane + 32 i: row n = 64 * half + v / 2, k half h = v % 2
        // (four packed words, the 16-byte chunk (st % 4) * 2 + h of the row's
        // swizzled 128-byte box row -> four 16-byte chunks of the f16 row).
        const int dw = warp - kDqWarp0;
        const int slot = dw >> 1, half = dw & 1;
        for (int st = slot; st < L.stages; st += kAStages) {
            if (!mbar_wait(raw_full(st >> 2), 0u, abort_flag, status, kStatusTimeoutDequant)) break;
            if (st >= kAStages && !mbar_wait(stage_done(st - kAStages), 0u, abort_flag, status, kStatusTimeoutDequant))
                break;
            const uint8_t* raw = smem + L.raw_off + (st >> 2) * L.raw_box;
            const uint32_t atile = base + L.a_off + slot * kRows * 128;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int v = lane + 32 * i;
                const int n = half * 64 + (v >> 1), h = v & 1;
                if (n < box_rows) {  // rows past the box stay stale; their TMEM lanes are never read
                    const int chunk = (((st & 3) * 2 + h) ^ (n & 7));
                    const uint4 q = *reinterpret_cast<const uint4*>(raw + n * 128 + chunk * 16);
                    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        sts128(atile + n * 128 + ((static_cast<uint32_t>(h * 4 + j) ^ static_cast<uint32_t>(n & 7)) << 4),
                               unpack_word_f16_perm(words[j]));
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(a_full(slot));
        }
    } else if (warp >= kEpWarp0) {
        // ------------------------------------------------- B tile, epilogue --
        const int et = tid - kEpWarp0 * 32;  // 0..127
        const int ew = warp - kEpWarp0;
        bool ok = mbar_wait(x_full, 0u, abort_flag, status, kStatusTimeoutEpilogue);
        const float* xs = reinterpret_cast<const float*>(smem + L.x_off);
        // items (stage, word): 8 consecutive k of the slice
        const int items = L.stages * 8;
        float mx[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) mx[m] = 0.0f;
        if (ok) {
            for (int it = et; it < items; it += 128) {
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    if (m < M) {
                        const float4 a = *reinterpret_cast<const float4*>(xs + m * L.kslice + it * 8);
                        const float4 b = *reinterpret_cast<const float4*>(xs + m * L.kslice + it * 8 + 4);
                        mx[m] = fmaxf(mx[m], fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
                        mx[m] = fmaxf(mx[m], fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx[m] = fmaxf(mx[m], __shfl_xor_sync(0xffffffffu, mx[m], off));
        }
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < 8; ++m) row_max[ew * 8 + m] = mx[m];
        }
        epilogue_sync();
        float rs[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const float v = fmaxf(fmaxf(row_max[m], row_max[8 + m]), fmaxf(row_max[16 + m], row_max[24 + m]));
            const int e = row_exponent(v);
            rs[m] = exp2i(e);
            if (et == 0) row_exp[m] = e;
        }
        if (ok) {
            for (int it = et; it < items; it += 128) {
                const int st = it >> 3, w = it & 7;
                const uint32_t tile = base + L.b_off + st * 16 * 128;
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    float v[8];
                    if (m < M) {
                        const float4 a = *reinterpret_cast<const float4*>(xs + m * L.kslice + it * 8);
                        const float4 b = *reinterpret_cast<const float4*>(xs + m * L.kslice + it * 8 + 4);
                        v[0] = a.x * rs[m]; v[1] = a.y * rs[m]; v[2] = a.z * rs[m]; v[3] = a.w * rs[m];
                        v[4] = b.x * rs[m]; v[5] = b.y * rs[m]; v[6] = b.z * rs[m]; v[7] = b.w * rs[m];
                    } else {
#pragma unroll
                        for (int i = 0; i < 8; ++i) v[i] = 0.0f;
                    }
                    uint32_t hw[4], lw[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {  // pair (k = i, k = i + 4)
                        const __half2 hh = __floats2half2_rn(v[i], v[i + 4]);
                        const float2 hf = __half22float2(hh);
                        const __half2 ll = __floats2half2_rn(v[i] - hf.x, v[i + 4] - hf.y);
                        hw[i] = *reinterpret_cast<const uint32_t*>(&hh);
                        lw[i] = *reinterpret_cast<const uint32_t*>(&ll);
                    }
                    // rows m (hi) and 8 + m (lo); chunk w swizzled by row & 7 (= m)
                    const uint32_t chunk = (static_cast<uint32_t>(w) ^ static_cast<uint32_t>(m)) << 4;
                    sts128(tile + m * 128 + chunk, make_uint4(hw[0], hw[1], hw[2], hw[3]));
                    sts128(tile + (8 + m) * 128 + chunk, make_uint4(lw[0], lw[1], lw[2], lw[3]));
                }
            }
        }
        fence_proxy_async_smem();
        epilogue_sync();
        if (et == 0) mbar_arrive(b_ready);

        float acc[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) acc[m] = 0.0f;
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll
        for (int gi = 0; gi < kMaxGroups; ++gi) {
            if (gi < L.groups && ok) {
                if (!mbar_wait(stage_done(gi >> 1), 0u, abort_flag, status, kStatusTimeoutEpilogue)) {
                    ok = false;
                } else {
                    tc_fence_after_sync();
                    uint32_t r[16];
                    tmem_ld16(lane_base + static_cast<uint32_t>(gi * kSlotCols), r);
                    tmem_ld_wait();
#pragma unroll
                    for (int m = 0; m < 8; ++m)
                        acc[m] = fmaf(sc[gi], __uint_as_float(r[m]) + __uint_as_float(r[8 + m]), acc[m]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) part[col * 8 + m] = acc[m] * exp2i(-row_exp[m]);
    }

    // ------------------------------------- cross-slice sum, LoRA, store --
    pdl_wait();  // T and Y may be touched by the previous launch (returns at once by now)
    tc_fence_before_sync();
    if (S > 1) {
        cluster_sync_all();
    } else {
        __syncthreads();
    }
    if (*abort_flag == 0) {
        cg::cluster_group cluster = cg::this_cluster();
        const int c_lo = C * crank / S, c_hi = C * (crank + 1) / S;  // columns this CTA finishes
        for (int idx = tid; idx < (c_hi - c_lo) * M; idx += kThreads) {
            const int cl = c_lo + idx / M, m = idx % M;
            const int n = n0 + cl;
            if (n >= N) continue;
            float v[8];
#pragma unroll
            for (int r = 0; r < 8; ++r) v[r] = r < S ? cluster.map_shared_rank(part, r)[cl * 8 + m] : 0.0f;
            float sum = v[0];
#pragma unroll
            for (int r = 1; r < 8; ++r) sum += v[r];  // fixed rank order; ranks >= S add zero
            if (lora_b != nullptr) {
                float d = 0.0f;
                for (int j = 0; j < rank; ++j) d = fmaf(lora_t[m * rank + j], lora_b[static_cast<size_t>(j) * N + n], d);
                sum = fmaf(lora_scale, d, sum);
            }
            y[static_cast<size_t>(m) * N + n] = sum;
        }
    } else if (warp == 0 && lane == 0) {
        // copies already issued land before the CTA's shared memory is released
        for (int b = 0; b < L.boxes; ++b) mbar_drain(raw_full(b), 0u);
        mbar_drain(x_full, 0u);
    }
    if (S > 1) cluster_sync_all();  // partials stay alive until every peer has read them
    if (warp == 1) {
        mbar_drain(mma_done, 0u);  // no MMA may still write the TMEM being freed
        tc_fence_after_sync();
        tmem_dealloc(tmem_base, kMaxGroups * kSlotCols);
    }
}

int max_clusters_cache[9][2] = {};  // [S][0] = smem bytes cached for, [S][1] = clusters

}  // namespace

size_t decode_smem_bytes(int M, int K, int S, int box_rows) {
    return static_cast<size_t>(decode_layout(M, K, S, box_rows).bytes);
}

// K split: the smallest S (cluster size) leaving <= 1024 k (32 groups) per CTA;
// 0 when the shape is not supported.
int decode_split(int M, int K) {
    if (M < 1 || M > 8 || K % kXBox != 0) return 0;
    for (int S = 1; S <= 8; S *= 2)
        if (K % (S * kRawBoxK) == 0 && K / S <= kMaxGroups * 32) return S;
    return 0;
}

int decode_max_clusters(int M, int K, int S, int box_rows) {
    const size_t smem = decode_smem_bytes(M, K, S, box_rows);
    if (smem > 227 * 1024 || S < 1 || S > 8) return 0;
    int (&c)[2] = max_clusters_cache[S];
    if (c[0] == static_cast<int>(smem)) return c[1];
    cudaError_t e = cudaFuncSetAttribute(q4_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(S));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(S);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, q4_decode_kernel, &cfg) != cudaSuccess) return 0;
    c[0] = static_cast<int>(smem);
    c[1] = n;
    return n;
}

int decode_rows() { return kRows; }
int decode_x_box() { return kXBox; }

int launch_decode(const DecodeArgs& a, cudaStream_t stream) {
    const int S = a.cluster_k;
    if (decode_split(a.M, a.K) != S || a.col_blocks < 1 || a.box_rows < 8 || a.box_rows > kRows ||
        (a.N + a.col_blocks - 1) / a.col_blocks > a.box_rows)
        return static_cast<int>(cudaErrorInvalidValue);
    const size_t smem = decode_smem_bytes(a.M, a.K, S, a.box_rows);
    cudaError_t e =
        cudaFuncSetAttribute(q4_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(S * a.col_blocks), 1, 1);
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
    e = cudaLaunchKernelEx(&cfg, q4_decode_kernel, a.tmap_w, a.tmap_x, a.scales, a.y, a.M, a.N, a.K, a.col_blocks,
                           a.box_rows, a.lora_t, a.lora_b, a.rank, a.lora_scale, a.status);
    return static_cast<int>(e);
}

}  // namespace q4
