// Decode GEMV, whole tile resident (M <= 8):  Y[M x N] = X . dequant(W) (+ LoRA), fp32.
//
// Same math and weight layout as the reference kernel (q4gemm.comp:7-19,
// 104-122): nibble v of column n at byte n*(K/2) + k/2 (low nibble = even k),
// w = float(v) * scales[n*(K/32) + k/32], y = sum_k x * w, all fp32.  The
// reference itself has no decode path (q4gemm.comp:36-37 needs M % 64 == 0).
//
// Designed for the latency of one small layer (4096 x 4096 int4 is 10.5 MB,
// ~1.6 us of HBM time): nothing waits on anything but the arrival of data.
//   * A CTA owns 32 columns and a K slice (the whole of K, or 1/S of it with a
//     cluster of S CTAs).  At entry one thread issues every TMA load of the
//     CTA's tile into its own shared memory: the packed weights as 128-byte
//     swizzled boxes of 32 columns x 256 k (one mbarrier per box), the scales
//     as swizzled boxes of 32 columns x 32 groups.  These do not depend on the
//     previous launch, so they go out before griddepcontrol.wait, and the CTA
//     signals its dependents at once: the next layer's CTAs can stream their
//     weights while this layer computes.  X (after the wait) is one TMA box
//     per row.
//   * The warps take the weight boxes round robin.  Lane (cq = lane/4, j =
//     lane%4) handles columns cq, cq+8, cq+16, cq+24 and, in each 32-k scale
//     group, the 8 k of word j: the weights are unpacked exactly (2^23 magic
//     number), scaled in fp32 (the reference's single rounding) and multiplied
//     into packed f32x2 accumulators; one x load serves four columns.  With the
//     swizzle every shared-memory load is free of bank conflicts.
//   * lanes j are summed with two shuffles, warps through shared memory, the
//     cluster's K slices through distributed shared memory, all in a fixed
//     order (deterministic).  The LoRA term (alpha/r) * T[m,:] . B[:,n] with
//     T = X*A is added and Y stored.
// No TMEM, no producer/consumer ring: the only waits are for TMA arrivals,
// each bounded (status word + abort flag).
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "common.cuh"
#include "q4_dequant.cuh"
#include "q4_kernels.h"

namespace cg = cooperative_groups;

namespace q4 {

namespace {

constexpr int kTSlot = 32;       // rows (columns of W) per shared-memory box slot
constexpr int kTBoxK = 256;      // k per weight box: one 128-byte row (32 words) per column
constexpr int kTScaleBoxG = 32;  // scale groups per scale box: one 128-byte row per column

// Warps per CTA: 8 on the fp32 path (M <= 3; each warp takes two or more
// weight boxes and has up to 128 registers, enough independent work to hide
// latency: 4.36 / 5.36 / 7.81 us per layer at M = 1 / 2 / 3 against 4.50 /
// 5.61 / 8.08 with 16 warps and 4.61 / 5.78 with 4), 16 on the mma path (its
// X conversion spreads each row over 512 threads).  At M <= 2 two CTAs share
// an SM.
template <int M>
struct TileCfg {
    // M >= 4 multiplies on the tensor cores with mma.sync (see below): its
    // loop costs the same at every M (3.3 us per layer in a 24-layer graph at
    // K = N = 4096), but every CTA first converts all of X into f16 hi/lo
    // planes (1.4 us at M = 4, 2.1 us at M = 8).  Against the fp32 path (M
    // FMAs per weight: 5.0 us at M = 4) it is ahead from M = 4 on: 8.70
    // against 8.93 us per layer there, and M = 3 stays on the fp32 path
    // (8.08 us).
    static constexpr bool kMma = M >= 4;
    static constexpr int kWarps = M <= 3 ? 8 : 16;
    static constexpr int kThreads = kWarps * 32;
    // X conversion of the mma path: float4 per thread and row (M * kslice <= 32768)
    static constexpr int kConvPerRow = (16 + M - 1) / M;
};

__host__ __device__ inline int tile_warps(int M) { return M <= 3 ? 8 : 16; }

// Test hook (gemv_tile_set_wait_test): when set, warp 0 of every CTA also
// waits for a second phase of its first weight barrier, which nothing arms,
// so that bounded wait runs out and the timeout path runs (status word,
// abort flag, the CTA returns).  Read once per warp-0 thread at entry.
static __device__ int g_tile_stall_test = 0;

struct TileLayout {
    int kslice, nbox, nsbox;
    int w_off, s_off, x_off, x_bytes, part_off, cpart_off, bar_off, misc_off, bytes;
};

__host__ __device__ inline TileLayout tile_layout(int M, int K, int S) {
    TileLayout L;
    L.kslice = K / S;
    L.nbox = L.kslice / kTBoxK;
    L.nsbox = (L.kslice / 32 + kTScaleBoxG - 1) / kTScaleBoxG;
    L.w_off = 0;                                       // nbox x [32 rows][128 B], swizzled
    L.s_off = L.w_off + L.nbox * kTSlot * 128;        // nsbox x [32 rows][128 B], swizzled
    L.x_off = L.s_off + L.nsbox * kTSlot * 128;       // [M][kslice] fp32
    // the per-warp partials [warp][M][32] reuse the X region once X is consumed
    const int part_bytes = tile_warps(M) * kTSlot * M * 4;
    L.x_bytes = M * L.kslice * 4 > part_bytes ? M * L.kslice * 4 : part_bytes;
    L.part_off = L.x_off;
    L.cpart_off = L.x_off + L.x_bytes;                 // [M][32] fp32 (the CTA's K-slice sum)
    L.bar_off = L.cpart_off + kTSlot * M * 4;
    L.misc_off = L.bar_off + (L.nbox + 2) * 8;         // wfull[nbox], sfull, xfull
    // abort flag; then (mma path) row-max scratch [16 warps][8] and row exponents [8]
    L.bytes = L.misc_off + 16 + 16 * 8 * 4 + 8 * 4;
    return L;
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}

// 2-D TMA load with an L2 evict-first policy (streamed-once weights).
__device__ __forceinline__ void tma_load_2d_stream(uint32_t dst, const void* tmap, uint32_t bar, int32_t c0,
                                                   int32_t c1, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// The eight int4 values of one packed word (k = 0..7 at bits 4k) as four
// f32x2 pairs (k, k+1), exactly: (u ^ 8) = v + 8 lies in [0, 15] and
// float(0x4B000000 | (v + 8)) = 2^23 + v + 8, so subtracting 2^23 + 8 gives v.
__device__ __forceinline__ void unpack_word_f32(uint32_t q, float2 (&v)[4]) {
    const uint32_t lo = (q ^ 0x88888888u) & 0x0F0F0F0Fu;         // k = 0, 2, 4, 6
    // q >> 4 as the high word of q * 2^28 (an integer multiply, off the
    // logic pipe that the byte permutes below saturate)
    const uint32_t hi = (__umulhi(q, 1u << 28) ^ 0x08080808u) & 0x0F0F0F0Fu;  // k = 1, 3, 5, 7
    const float2 nbias = make_float2(-8388616.0f, -8388616.0f);                 // -(2^23 + 8)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        // byte_perm selector 0x744b: byte b -> byte 0, zeros -> bytes 1-2,
        // 0x4B (the exponent byte of 2^23) -> byte 3.
        const float2 mg = make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b))),
                                      __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b))));
        v[b] = __fadd2_rn(mg, nbias);
    }
}

// The same eight weights times the group scale: float(v) * s rounded once, as
// the reference's dequant.
__device__ __forceinline__ void dequant_word_f32(uint32_t q, float s, float2 (&w)[4]) {
    float2 v[4];
    unpack_word_f32(q, v);
    const float2 s2 = make_float2(s, s);
#pragma unroll
    for (int b = 0; b < 4; ++b) w[b] = __fmul2_rn(v[b], s2);
}

template <int M>
__global__ void __launch_bounds__(TileCfg<M>::kThreads, (M <= 2 ? 2 : 1))
    q4_gemv_tile_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_s,
                        const __grid_constant__ CUtensorMap tmap_x, float* __restrict__ y, int N, int K, int G,
                        const float* __restrict__ lora_t, const float* __restrict__ lora_b, int rank,
                        float lora_scale, int* __restrict__ status) {
    constexpr int kWarps = TileCfg<M>::kWarps;
    constexpr int kThreads = TileCfg<M>::kThreads;
    extern __shared__ uint8_t smem_raw[];
    // 128-byte swizzled TMA destinations need 1024-byte alignment.
    // 128-byte swizzled TMA boxes need 1024-byte alignment in the shared
    // window; dynamic shared memory of a kernel without static shared memory
    // starts 1024-aligned.  Anything else is reported, not used.
    uint8_t* smem = smem_raw;
    const uint32_t base = smem_u32(smem_raw);
    if ((base & 1023u) != 0) {
        if (threadIdx.x == 0 && status) atomicCAS(status, 0, kStatusBadLaunch);
        return;
    }
    const int S = static_cast<int>(cluster_nctarank());
    const int crank = static_cast<int>(cluster_ctarank());
    const TileLayout L = tile_layout(M, K, S);
    // Column block blk of G: columns [blk*N/G, (blk+1)*N/G), at most 32.  The
    // boxes load ceil(N/G) rows from n0; a row past the block belongs to the
    // next block (or lies past N, zero-filled) and is never stored.
    const int blk = static_cast<int>(blockIdx.x) / S;
    const int n0 = static_cast<int>(static_cast<long long>(blk) * N / G);
    const int C = static_cast<int>(static_cast<long long>(blk + 1) * N / G) - n0;
    const int box_rows = (N + G - 1) / G;
    const int k0 = crank * L.kslice;

    const uint32_t bar = base + L.bar_off;
    auto wfull = [&](int b) { return bar + 8u * b; };
    const uint32_t sfull = bar + 8u * L.nbox;
    const uint32_t xfull = bar + 8u * (L.nbox + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int stall_test = warp == 0 ? *static_cast<volatile int*>(&g_tile_stall_test) : 0;
    if (tid == 0) {
        for (int b = 0; b < L.nbox + 2; ++b) mbar_init(bar + 8u * b, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    __syncthreads();

    if (tid == 0) {
        // Weights and scales do not depend on the previous launch.
        tma_prefetch_desc(&tmap_w);
        tma_prefetch_desc(&tmap_s);
        tma_prefetch_desc(&tmap_x);
        const uint64_t pol = policy_evict_first();
        // boxes are C rows; each lands in a 32-row (4 KB) slot
        mbar_arrive_expect_tx(sfull, static_cast<uint32_t>(L.nsbox * box_rows * 128));
        for (int sb = 0; sb < L.nsbox; ++sb)
            tma_load_2d_stream(base + L.s_off + sb * kTSlot * 128, &tmap_s, sfull, k0 / 32 + sb * kTScaleBoxG, n0,
                               pol);
        for (int b = 0; b < L.nbox; ++b) {
            mbar_arrive_expect_tx(wfull(b), static_cast<uint32_t>(box_rows * 128));
            tma_load_2d_stream(base + L.w_off + b * kTSlot * 128, &tmap_w, wfull(b), (k0 + b * kTBoxK) / 8, n0, pol);
        }
    }
    // Dependents may launch now: their weight loads overlap this launch.
    pdl_launch_dependents();
    pdl_wait();  // X, T and Y may be touched by the previous launch
    if (tid == 0) {
        mbar_arrive_expect_tx(xfull, static_cast<uint32_t>(M * L.kslice * 4));
        const int rows_per_m = K / kTBoxK;
        for (int m = 0; m < M; ++m)
            tma_load_2d(base + L.x_off + m * L.kslice * 4, &tmap_x, xfull, 0, m * rows_per_m + k0 / kTBoxK);
    }

    if constexpr (TileCfg<M>::kMma) {
        // ---------------------------------------------- compute (mma path) --
        // Warp-level tensor-core MMA (mma.sync m16n8k16, f16 in, fp32
        // accumulate), issued from registers: no TMEM, no commits.
        //   A (16 x 16): rows 0-7 = x_hi of rows 0-7, rows 8-15 = x_lo, with
        //   x * 2^e_m = x_hi + x_lo (f16, e_m per row and K slice);
        //   B (16 x 8): 8 weight columns, the int4 values v as f16 (exact);
        //   D[g][n] + D[g + 8][n] = 2^e_g * sum_k x[g][k] v[k][n] over 16 k.
        // Two MMAs per 32-k scale group into a fresh D, then y += s(n, g) * D
        // in fp32.  The thread of lane (g = lane / 4, q = lane % 4) owns x-row g
        // and columns 8o + 2q, 8o + 2q + 1 of each column octet o.
        bool ok = mbar_wait(sfull, 0u, abort_flag, status, kStatusTimeoutGemv) &&
                  mbar_wait(xfull, 0u, abort_flag, status, kStatusTimeoutGemv);
        if (stall_test)  // phase 0 of box 0's barrier completes; phase 1 is never armed
            ok = ok && mbar_wait(wfull(0), 0u, abort_flag, status, kStatusTimeoutGemv) &&
                 mbar_wait(wfull(0), 1u, abort_flag, status, kStatusTimeoutGemv);
        uint32_t* rmax = reinterpret_cast<uint32_t*>(smem + L.misc_off + 16);     // [16 warps][8], float bits
        int* rexp = reinterpret_cast<int*>(smem + L.misc_off + 16 + 16 * 8 * 4);    // [8]
        // X -> per-row exponents and f16 hi/lo planes, in place.  Thread t
        // takes float4 t, t + 512, ... of each row (consecutive threads,
        // consecutive 16 bytes), keeps them in registers for the row maxima
        // (|x| as bits: unsigned order = float order; one redux per row and
        // warp), and after two barriers writes each as 8 bytes of the planes,
        // with 8-k chunk c of row m at position c ^ (m & 7).
        constexpr int kPerRow = TileCfg<M>::kConvPerRow;  // float4 per thread and row
        const int f4_row = L.kslice / 4;
        float4 xv[M][kPerRow];
        const float4* xf = reinterpret_cast<const float4*>(smem + L.x_off);
#pragma unroll
        for (int m = 0; m < M; ++m) {
            uint32_t mb = 0;
#pragma unroll
            for (int i = 0; i < kPerRow; ++i) {
                const int f = tid + i * kThreads;
                xv[m][i] = (f < f4_row && ok) ? xf[m * f4_row + f] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                const uint32_t a = __float_as_uint(fmaxf(fmaxf(fabsf(xv[m][i].x), fabsf(xv[m][i].y)),
                                                         fmaxf(fabsf(xv[m][i].z), fabsf(xv[m][i].w))));
                mb = a > mb ? a : mb;
            }
            mb = __reduce_max_sync(0xffffffffu, mb);
            if (lane == 0) rmax[warp * 8 + m] = mb;
        }
        __syncthreads();  // every warp's row maxima are out; X is in registers
        if (tid < M) {
            uint32_t vb = 0;
            for (int w16 = 0; w16 < kWarps; ++w16) vb = rmax[w16 * 8 + tid] > vb ? rmax[w16 * 8 + tid] : vb;
            const float v = __uint_as_float(vb);
            int e = 0;
            if (v > 0.0f && isfinite(v)) {
                int e2;
                frexpf(v, &e2);
                e = 14 - e2;  // max|x| * 2^e in [2^13, 2^14)
                e = e < -60 ? -60 : (e > 60 ? 60 : e);
            }
            rexp[tid] = e;
        }
        __syncthreads();
        uint8_t* hi_plane = smem + L.x_off;
        uint8_t* lo_plane = hi_plane + M * L.kslice * 2;
        const int cpr = L.kslice / 8;  // 8-k chunks per row
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float sc = exp2i(rexp[m]);
            const float2 sc2 = make_float2(sc, sc);
#pragma unroll
            for (int i = 0; i < kPerRow; ++i) {
                const int f = tid + i * kThreads;
                if (f < f4_row && ok) {
                    const float2 a01 = __fmul2_rn(make_float2(xv[m][i].x, xv[m][i].y), sc2);
                    const float2 a23 = __fmul2_rn(make_float2(xv[m][i].z, xv[m][i].w), sc2);
                    const __half2 h01 = __float22half2_rn(a01), h23 = __float22half2_rn(a23);
                    const float2 b01 = __half22float2(h01), b23 = __half22float2(h23);
                    const float2 r01 = __fadd2_rn(a01, make_float2(-b01.x, -b01.y));
                    const float2 r23 = __fadd2_rn(a23, make_float2(-b23.x, -b23.y));
                    const __half2 l01 = __float22half2_rn(r01), l23 = __float22half2_rn(r23);
                    const int c = f >> 1;
                    const int pos = (m * cpr + (c ^ (m & 7))) * 16 + (f & 1) * 8;
                    *reinterpret_cast<uint2*>(hi_plane + pos) =
                        make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
                    *reinterpret_cast<uint2*>(lo_plane + pos) =
                        make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
                }
            }
        }
        __syncthreads();

        const int g = lane >> 2, q = lane & 3;
        const int mrow = g < M ? g : M - 1;  // A rows past M repeat a row; their D rows are never stored
        // plain C++ loads (ordered after the mbarrier waits, free to be scheduled)
        const uint8_t* hi_row = smem + L.x_off + mrow * L.kslice * 2 + q * 4;
        const uint8_t* lo_row = hi_row + M * L.kslice * 2;
        const uint32_t msw = static_cast<uint32_t>(mrow & 7);
        const uint32_t bsel = 0x4040u | (static_cast<uint32_t>(q) << 8) | static_cast<uint32_t>(q);  // byte q, twice
        const __half2 vmul = __halves2half2(__ushort_as_half(0x3C00u), __ushort_as_half(0x2C00u));  // 1, 1/16
        const __half2 vadd = __halves2half2(__ushort_as_half(0xE408u), __ushort_as_half(0xD480u));  // -1032, -72
        float accm[4][2];
#pragma unroll
        for (int o = 0; o < 4; ++o) accm[o][0] = accm[o][1] = 0.0f;
#pragma unroll 1
        for (int b = warp; b < L.nbox && ok; b += kWarps) {
            if (!mbar_wait(wfull(b), 0u, abort_flag, status, kStatusTimeoutGemv)) {
                ok = false;
                break;
            }
            const uint8_t* wcol = smem + L.w_off + b * kTSlot * 128 + g * 128;  // column 8o + g at + o * 1024
            const uint8_t* sbx = smem + L.s_off + (b >> 2) * kTSlot * 128;
            const int schunk0 = (b & 3) * 2;
#pragma unroll  // all eight groups in flight: 3.26 against 3.6 us per layer with two (M = 8, in the graph)
            for (int t = 0; t < 8; ++t) {
                // A fragments of this 32-k group: chunks c0 .. c0 + 3 of the row
                const uint32_t c0 = static_cast<uint32_t>(b * 32 + t * 4);
                uint32_t a[2][4];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t ca = ((c0 + 2 * h) ^ msw) << 4, cb = ((c0 + 2 * h + 1) ^ msw) << 4;
                    a[h][0] = *reinterpret_cast<const uint32_t*>(hi_row + ca);
                    a[h][1] = *reinterpret_cast<const uint32_t*>(lo_row + ca);
                    a[h][2] = *reinterpret_cast<const uint32_t*>(hi_row + cb);
                    a[h][3] = *reinterpret_cast<const uint32_t*>(lo_row + cb);
                }
#pragma unroll
                for (int o = 0; o < 4; ++o) {
                    // column 8o + g: its 16-byte word of group t (swizzle key g)
                    const uint4 wq = *reinterpret_cast<const uint4*>(
                        wcol + o * 1024 + ((static_cast<uint32_t>(t) ^ static_cast<uint32_t>(g)) << 4));
                    const uint32_t words[4] = {wq.x, wq.y, wq.z, wq.w};
                    uint32_t bf[4];
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        // byte q of word w: nibbles k = 8w + 2q, 8w + 2q + 1 -> f16 pair (exact)
                        const uint32_t both = __byte_perm(words[w], 0u, bsel);
                        const uint32_t tt = ((both ^ 0x00800008u) & 0x00F0000Fu) | 0x64006400u;
                        const __half2 v = __hfma2(*reinterpret_cast<const __half2*>(&tt), vmul, vadd);
                        bf[w] = *reinterpret_cast<const uint32_t*>(&v);
                    }
                    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        asm(
                            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
                            "{%8,%9}, {%0,%1,%2,%3};"
                            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                            : "r"(a[h][0]), "r"(a[h][1]), "r"(a[h][2]), "r"(a[h][3]), "r"(bf[2 * h]), "r"(bf[2 * h + 1]));
                    }
                    // scales of columns 8o + 2q and 8o + 2q + 1 (swizzle key 2q + e)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const uint32_t cc = static_cast<uint32_t>(o * 8 + 2 * q + e);
                        const float sv = *reinterpret_cast<const float*>(
                            sbx + cc * 128 + (((static_cast<uint32_t>(schunk0 + (t >> 2))) ^ (cc & 7u)) << 4) + (t & 3) * 4);
                        accm[o][e] = fmaf(sv, d[e] + d[2 + e], accm[o][e]);
                    }
                }
            }
        }
        // ------------------------------------------------------------- reduce --
        __syncthreads();  // every warp is done with X: its region takes the partials
        float* part = reinterpret_cast<float*>(smem + L.part_off);  // [warp][M][col]
        if (g < M) {
            const float unscale = exp2i(-rexp[g]);
#pragma unroll
            for (int o = 0; o < 4; ++o)
#pragma unroll
                for (int e = 0; e < 2; ++e) part[(warp * M + g) * kTSlot + o * 8 + 2 * q + e] = accm[o][e] * unscale;
        }
        __syncthreads();
    } else {
        // ------------------------------------------------- compute (fp32 path) --
        // Lane (cq, j) handles slot rows cq + 8r (r < 4) and word j of each group;
        // rows >= C (C < 32) hold no column and their sums are never read.  All
        // four rows of a lane share row & 7 = cq, so in the 128-byte swizzle the
        // 16-byte chunk of group t is t ^ cq for every r: one LOP3 per group
        // addresses the four words (and another the four scales), and the eight
        // lanes cq of a quarter warp hit distinct bank quads.
        const int cq = lane >> 2, j = lane & 3;
        const uint32_t cq16 = static_cast<uint32_t>(cq) << 4;
        float2 acc[4][M];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int m = 0; m < M; ++m) acc[r][m] = make_float2(0.0f, 0.0f);

        bool ok = mbar_wait(sfull, 0u, abort_flag, status, kStatusTimeoutGemv) &&
                  mbar_wait(xfull, 0u, abort_flag, status, kStatusTimeoutGemv);
        if (stall_test)  // phase 0 of box 0's barrier completes; phase 1 is never armed
            ok = ok && mbar_wait(wfull(0), 0u, abort_flag, status, kStatusTimeoutGemv) &&
                 mbar_wait(wfull(0), 1u, abort_flag, status, kStatusTimeoutGemv);
        const uint32_t xs = base + L.x_off + j * 32;  // this lane's 8 x of word j in a group
#pragma unroll 1
        for (int b = warp; b < L.nbox && ok; b += kWarps) {
            if (!mbar_wait(wfull(b), 0u, abort_flag, status, kStatusTimeoutGemv)) {
                ok = false;
                break;
            }
            // bits 4-6 of both bases are zero, so "| chunk << 4" places the chunk
            const uint32_t wrow = base + L.w_off + b * kTSlot * 128 + cq * 128 + j * 4;
            const uint32_t srow = base + L.s_off + (b >> 2) * kTSlot * 128 + cq * 128;
            const uint32_t sx = (static_cast<uint32_t>((b & 3) * 2) << 4) ^ cq16;  // scale chunk of group 0, swizzled
            const uint32_t xrow = xs + b * kTBoxK * 4;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const uint32_t wa = wrow | ((static_cast<uint32_t>(t) << 4) ^ cq16);
                const uint32_t sa = (srow | (sx ^ (static_cast<uint32_t>(t >> 2) << 4))) + (t & 3) * 4;
                if constexpr (M <= 2) {
                    float2 xv[M][4];
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        const float4 xa = lds_f4(xrow + m * L.kslice * 4 + t * 128);
                        const float4 xc = lds_f4(xrow + m * L.kslice * 4 + t * 128 + 16);
                        xv[m][0] = make_float2(xa.x, xa.y);
                        xv[m][1] = make_float2(xa.z, xa.w);
                        xv[m][2] = make_float2(xc.x, xc.y);
                        xv[m][3] = make_float2(xc.z, xc.w);
                    }
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const uint32_t q = lds_u32(wa + r * 8 * 128);
                        const float s = __uint_as_float(lds_u32(sa + r * 8 * 128));
                        // per-word partial sum of v * x, scaled once (fewer fp32 ops)
                        float2 v[4];
                        unpack_word_f32(q, v);
#pragma unroll
                        for (int m = 0; m < M; ++m) {
                            float2 p = __fmul2_rn(v[0], xv[m][0]);
                            p = __ffma2_rn(v[1], xv[m][1], p);
                            p = __ffma2_rn(v[2], xv[m][2], p);
                            p = __ffma2_rn(v[3], xv[m][3], p);
                            acc[r][m].x = fmaf(s, p.x + p.y, acc[r][m].x);
                        }
                    }
                } else {
                    // the four columns' scaled weights first, then X one row at a
                    // time: 32 + 8 live registers besides the accumulators
                    float2 w[4][4];
#pragma unroll
                    for (int r = 0; r < 4; ++r)
                        dequant_word_f32(lds_u32(wa + r * 8 * 128), __uint_as_float(lds_u32(sa + r * 8 * 128)), w[r]);
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        const float4 xa = lds_f4(xrow + m * L.kslice * 4 + t * 128);
                        const float4 xc = lds_f4(xrow + m * L.kslice * 4 + t * 128 + 16);
                        const float2 x0 = make_float2(xa.x, xa.y), x1 = make_float2(xa.z, xa.w);
                        const float2 x2 = make_float2(xc.x, xc.y), x3 = make_float2(xc.z, xc.w);
#pragma unroll
                        for (int r = 0; r < 4; ++r) {
                            acc[r][m] = __ffma2_rn(w[r][0], x0, acc[r][m]);
                            acc[r][m] = __ffma2_rn(w[r][1], x1, acc[r][m]);
                            acc[r][m] = __ffma2_rn(w[r][2], x2, acc[r][m]);
                            acc[r][m] = __ffma2_rn(w[r][3], x3, acc[r][m]);
                        }
                    }
                }
            }
        }

        // ------------------------------------------------------------- reduce --
        __syncthreads();  // every warp is done with X: its region takes the partials
        float* part = reinterpret_cast<float*>(smem + L.part_off);  // [warp][M][col]
#pragma unroll
        for (int r = 0; r < 4; ++r) {
#pragma unroll
            for (int m = 0; m < M; ++m) {
                float v = acc[r][m].x + acc[r][m].y;
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                if (j == 0) part[(warp * M + m) * kTSlot + cq + 8 * r] = v;
            }
        }
        __syncthreads();
    }

    const float* part = reinterpret_cast<const float*>(smem + L.part_off);  // [warp][M][col]
    float* cpart = reinterpret_cast<float*>(smem + L.cpart_off);  // [M][32]
    for (int idx = tid; idx < kTSlot * M; idx += kThreads) {
        float sum = 0.0f;
#pragma unroll
        for (int w8 = 0; w8 < kWarps; ++w8) sum += part[w8 * kTSlot * M + idx];
        cpart[idx] = sum;
    }
    if (S > 1) {
        cluster_sync_all();
    } else {
        __syncthreads();
    }
    cg::cluster_group cluster = cg::this_cluster();
    for (int idx = crank + S * tid; idx < kTSlot * M; idx += kThreads * S) {
        const int m = idx / kTSlot, c = idx % kTSlot;
        const int n = n0 + c;
        float sum = 0.0f;
        if (S > 1) {
            for (int q = 0; q < S; ++q) sum += cluster.map_shared_rank(cpart, q)[idx];
        } else {
            sum = cpart[idx];
        }
        if (c < C && n < N) {
            if (lora_b != nullptr) {
                float d = 0.0f;
                for (int jr = 0; jr < rank; ++jr) d = fmaf(lora_t[m * rank + jr], lora_b[static_cast<size_t>(jr) * N + n], d);
                sum = fmaf(lora_scale, d, sum);
            }
            y[static_cast<size_t>(m) * N + n] = sum;
        }
    }
    if (S > 1) cluster_sync_all();  // peers may still read this CTA's partials

    if (tid == 0 && *abort_flag) {
        // copies already issued land before the CTA's shared memory is released
        for (int b = 0; b < L.nbox; ++b) mbar_drain(wfull(b), 0u);
        mbar_drain(sfull, 0u);
        mbar_drain(xfull, 0u);
    }
}

template <int M>
int launch_tile_m(const GemvTileArgs& a, cudaStream_t stream) {
    const TileLayout L = tile_layout(M, a.K, a.cluster_k);
    const size_t smem = static_cast<size_t>(L.bytes);
    auto kern = q4_gemv_tile_kernel<M>;
    // The shared-memory allowance is set once per device (to the largest
    // layout this kernel takes), not per call: the attribute call costs about
    // a microsecond of host time, a fifth of a layer at M = 1.
    static std::atomic<bool> attr_done[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (dev < 0 || dev >= 64 || !attr_done[dev].load(std::memory_order_acquire)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return static_cast<int>(e);
        if (dev >= 0 && dev < 64) attr_done[dev].store(true, std::memory_order_release);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(a.col_blocks * a.cluster_k));
    cfg.blockDim = dim3(TileCfg<M>::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
    if (a.cluster_k > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = static_cast<unsigned>(a.cluster_k);
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    e = cudaLaunchKernelEx(&cfg, kern, a.tmap_w, a.tmap_s, a.tmap_x, a.y, a.N, a.K, a.col_blocks, a.lora_t, a.lora_b,
                           a.rank, a.lora_scale, a.status);
    return static_cast<int>(e);
}

}  // namespace

int gemv_tile_set_wait_test(unsigned long long limit_ns, int stall) {
    cudaError_t e = cudaMemcpyToSymbol(g_wait_limit_ns, &limit_ns, sizeof(limit_ns));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_tile_stall_test, &stall, sizeof(stall));
    return static_cast<int>(e);
}

size_t gemv_tile_smem_bytes(int M, int K, int S) { return static_cast<size_t>(tile_layout(M, K, S).bytes); }

bool gemv_tile_supported(int M, int K, int S) {
    if (M < 1 || M > 8 || S < 1 || S > 8 || (S & (S - 1)) != 0) return false;
    if (K <= 0 || K % (kTBoxK * S) != 0) return false;
    // the mma path (M >= 4) holds at most 16 float4 of X per thread while converting it
    if (M >= 4 && static_cast<long long>(M) * (K / S) > 16LL * 4 * 512) return false;
    return gemv_tile_smem_bytes(M, K, S) <= 227 * 1024;
}

// Column blocks: one per SM while that keeps blocks at <= 32 columns, so a
// launch holds exactly one CTA per SM and the next launch (programmatic
// dependent launch) finds exactly one free slot on every SM; wider matrices
// take 32-column blocks in several waves.  N = 4096 on 148 SMs: 148 blocks of
// 27 or 28 columns.
int gemv_tile_col_blocks(int N, int sm_count) {
    if (N <= 32 * sm_count) return N < sm_count ? N : sm_count;
    return (N + 31) / 32;
}

int gemv_tile_box_rows(int N, int col_blocks) { return (N + col_blocks - 1) / col_blocks; }

int gemv_tile_box_k() { return kTBoxK; }
int gemv_tile_scale_box_groups() { return kTScaleBoxG; }

int launch_gemv_tile(const GemvTileArgs& a, cudaStream_t stream) {
    if (!gemv_tile_supported(a.M, a.K, a.cluster_k) || a.col_blocks < 1 || a.col_blocks > a.N ||
        gemv_tile_box_rows(a.N, a.col_blocks) > kTSlot)
        return static_cast<int>(cudaErrorInvalidValue);
    switch (a.M) {
        case 1: return launch_tile_m<1>(a, stream);
        case 2: return launch_tile_m<2>(a, stream);
        case 3: return launch_tile_m<3>(a, stream);
        case 4: return launch_tile_m<4>(a, stream);
        case 5: return launch_tile_m<5>(a, stream);
        case 6: return launch_tile_m<6>(a, stream);
        case 7: return launch_tile_m<7>(a, stream);
        default: return launch_tile_m<8>(a, stream);
    }
}

}  // namespace q4
