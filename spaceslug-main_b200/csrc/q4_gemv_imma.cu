// Decode GEMV on the integer tensor cores (M <= 8):  Y[M x N] = X . dequant(W) (+ LoRA), fp32 result.
//
// Same weight layout and math as the reference kernel (q4gemm.comp:7-19,
// 104-122): nibble v of column n at byte n*(K/2) + k/2 (low nibble = even k),
// w = float(v) * scales[n*(K/32) + k/32], y = sum_k x * w.  The reference has
// no decode path (q4gemm.comp:36-37 needs M % 64 == 0).
//
// Exactness.  Per 32-k scale group g and column n the kernel forms the exact
// integer S = sum_k (16 v_k) * X'_k on the tensor cores, where X' is the row
// of X scaled by a power of two 2^e (per row and K slice, so that
// max |x| * 2^e lies in [2^21, 2^22)) and rounded to an integer, split into
// three signed 8-bit limbs X' = 2^16 h + 2^8 m + l (|h| <= 64).  The only
// rounding of X is that of X' to an integer: 2^-22 of the slice's largest
// |x|, below fp32 rounding of that element.  The weights enter as the exact
// signed bytes 16 v (the nibble moved to the byte's high half), so the
// products and the 32-term sums are exact in int32 (|S| < 2^19).  Each group
// sum is then scaled in fp32, y += s(n, g) * S, and the three limb sums are
// combined with their powers of two at the end.
//
//   * mma.sync.m16n8k32.s8.s8.s32: A = 16 weight columns x 32 k (thread (g, q)
//     holds word q of the group for columns g and g + 8: its even nibbles as
//     one register of four bytes, its odd nibbles as another -- the k order
//     inside the group is permuted the same way for X), B = 8 limb rows
//     (limb, row of X) x the same 32 k.  The accumulator input C is the bit
//     pattern of 1.5 * 2^23, so D read as a float is 1.5 * 2^23 + S exactly
//     (|S| < 2^22) and one FADD gives float(S): no int-to-float conversions.
//   * Work split.  A cluster of S CTAs splits K (each CTA converts and reads
//     only its K slice of X; the slices are summed through distributed shared
//     memory in a fixed order); a CTA owns T tiles of 16 columns, and its
//     T * P warps take one tile and one of P parts of the slice's groups.
//   * Loads.  At entry one thread issues TMA loads of the CTA's whole weight
//     and scale tile (128-byte swizzled boxes of 256 k x 16 T columns and
//     32 groups x 16 T columns), before griddepcontrol.wait: they do not
//     depend on the previous launch, the CTA signals its dependents at once,
//     and at <= ~100 KB of shared memory two CTAs share an SM, so the next
//     layer's weights stream while this layer computes.
// No TMEM and no producer/consumer ring: the only waits are for TMA arrivals,
// each bounded (status word + abort flag).
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "q4_dequant.cuh"
#include "q4_kernels.h"

namespace cg = cooperative_groups;

namespace q4 {

namespace {

constexpr int kIBoxK = 256;        // k per weight box: one 128-byte row (32 words) per column
constexpr int kIScaleBoxG = 32;    // scale groups per scale box: one 128-byte row per column
constexpr int kIMaxWarps = 16;
constexpr int kIMaxTiles = 7;      // 16-column tiles per CTA (shared-memory budget)
constexpr float kMagic = 12582912.0f;          // 1.5 * 2^23
constexpr int kMagicBits = 0x4B400000;

// Test hook (gemv_imma_set_wait_test): when set, warp 0 of every CTA also
// waits for a second phase of its first weight barrier, which nothing arms,
// so that bounded wait runs out and the timeout path runs.
static __device__ int g_imma_stall_test = 0;

struct ImmaLayout {
    int ks, gs, nbox, nsbox, rows, slots;
    int w_off, s_off, l_off, red_off, bar_off, misc_off, bytes;
    int part_off, cpart_off;  // alias the weight region once every warp is done with it
};

__host__ __device__ inline int imma_nb(int M) { return (3 * M + 7) / 8; }

__host__ __device__ inline ImmaLayout imma_layout(int M, int K, int S, int T, int P) {
    ImmaLayout L;
    L.ks = K / S;
    L.gs = L.ks / 32;
    L.nbox = L.ks / kIBoxK;
    L.nsbox = L.gs / kIScaleBoxG;
    L.rows = 16 * T;
    L.slots = 8 * imma_nb(M);
    L.w_off = 0;
    const int w_bytes = L.nbox * L.rows * 128;
    const int part_bytes = P * T * L.slots * 16 * 4;
    const int cpart_bytes = M * L.rows * 4;
    L.part_off = 0;
    L.cpart_off = (part_bytes + 127) / 128 * 128;
    const int region = w_bytes > L.cpart_off + cpart_bytes ? w_bytes : L.cpart_off + cpart_bytes;
    L.s_off = (region + 1023) / 1024 * 1024;                   // 128B-swizzled boxes: 1024-aligned
    L.l_off = L.s_off + L.nsbox * L.rows * 128;                // limb rows [slots][ks] bytes
    L.red_off = L.l_off + L.slots * L.ks;                      // row maxima [warps][8] u32, exps [8], bad [8]
    L.bar_off = L.red_off + (kIMaxWarps * 8 + 16) * 4;
    L.misc_off = L.bar_off + (L.nbox + L.nsbox) * 8;           // abort flag
    L.bytes = L.misc_off + 16;
    return L;
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ float ldsf(uint32_t addr) { return __uint_as_float(lds32(addr)); }
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ void sts64(uint32_t addr, uint32_t a, uint32_t b) {
    asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint64_t policy_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// D = A * B + D, int8 x int8 -> int32, m16n8k32 (A row-major, B column-major).
__device__ __forceinline__ void imma_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four bytes b0..b3 (byte 0 of each argument) into one word.
__device__ __forceinline__ uint32_t pack_bytes(uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3) {
    return __byte_perm(__byte_perm(b0, b1, 0x0040u), __byte_perm(b2, b3, 0x0040u), 0x5410u);
}

template <int NB>
__global__ void __launch_bounds__(kIMaxWarps * 32, 2)
    q4_gemv_imma_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_s,
                        const float* __restrict__ x, float* __restrict__ y, int M, int N, int K, int T, int P,
                        int tiles_total, int clusters, const float* __restrict__ lora_t,
                        const float* __restrict__ lora_b, int rank, float lora_scale, int* __restrict__ status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw;
    const uint32_t base = smem_u32(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nthreads = blockDim.x;
    const int W = nthreads >> 5;
    if ((base & 1023u) != 0) {  // 128B-swizzled TMA destinations need a 1024-aligned window
        if (tid == 0 && status) atomicCAS(status, 0, kStatusBadLaunch);
        return;
    }
    const int S = static_cast<int>(cluster_size());
    const int crank = static_cast<int>(cluster_ctarank());
    const ImmaLayout L = imma_layout(M, K, S, T, P);
    // cluster c owns tiles [c * tiles_total / clusters, (c + 1) * tiles_total / clusters)
    const int cl = static_cast<int>(blockIdx.x) / S;
    const int t0 = static_cast<int>(static_cast<long long>(cl) * tiles_total / clusters);
    const int t1 = static_cast<int>(static_cast<long long>(cl + 1) * tiles_total / clusters);
    const int n0 = 16 * t0;
    const int ncols = min(N, 16 * t1) - n0;  // columns this cluster stores (<= L.rows)
    const int k0 = crank * L.ks;
    const int stall_test = warp == 0 ? *static_cast<volatile int*>(&g_imma_stall_test) : 0;

    const uint32_t bar = base + L.bar_off;
    auto wfull = [&](int b) { return bar + 8u * b; };
    auto sfull = [&](int b) { return bar + 8u * (L.nbox + b); };
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off);
    uint32_t* red = reinterpret_cast<uint32_t*>(smem + L.red_off);  // [kIMaxWarps][8] row-max bits
    int* rexp = reinterpret_cast<int*>(red + kIMaxWarps * 8);        // [8] row exponents
    int* rbad = rexp + 8;                                            // [8] row holds a non-finite x

    if (tid == 0) {
        for (int b = 0; b < L.nbox + L.nsbox; ++b) mbar_init(bar + 8u * b, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    __syncthreads();
    if (tid == 0) {
        // weights and scales do not depend on the previous launch
        tma_prefetch_desc(&tmap_w);
        tma_prefetch_desc(&tmap_s);
        const uint64_t pol = policy_first();
        for (int b = 0; b < L.nsbox; ++b) {
            mbar_arrive_expect_tx(sfull(b), static_cast<uint32_t>(L.rows * 128));
            tma_load_2d_hint(base + L.s_off + b * L.rows * 128, &tmap_s, sfull(b), k0 / 32 + b * kIScaleBoxG, n0, pol);
        }
        for (int b = 0; b < L.nbox; ++b) {
            mbar_arrive_expect_tx(wfull(b), static_cast<uint32_t>(L.rows * 128));
            tma_load_2d_hint(base + L.w_off + b * L.rows * 128, &tmap_w, wfull(b), (k0 + b * kIBoxK) / 8, n0, pol);
        }
    }
    pdl_launch_dependents();  // the next launch's CTAs may start streaming their weights
    pdl_wait();               // X, T and Y may belong to the previous launch until here

    // ---------------------------------------------- X slice -> int8 limbs --
    // Chunk ch = (row m, 8 consecutive k of the slice).  Pass 1: row maxima.
    const int cpr = L.ks / 8;  // chunks per row
    const int nch = M * cpr;
    {
        float mx[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) mx[m] = 0.0f;
        for (int ch = tid; ch < nch; ch += nthreads) {
            const int m = ch / cpr, c = ch - m * cpr;
            const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(m) * K + k0 + 8 * c);
            const float4 a = src[0], b = src[1];
            // fmaxf drops NaN: a non-finite row is flagged through the sum below
            float cm = fmaxf(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))),
                             fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
            const float sum = a.x + a.y + a.z + a.w + b.x + b.y + b.z + b.w;
            if (!isfinite(sum) || !isfinite(cm)) cm = __int_as_float(0x7f800000);  // +inf marks the row
#pragma unroll
            for (int mm = 0; mm < 8; ++mm)
                if (mm == m) mx[mm] = fmaxf(mx[mm], cm);
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const uint32_t r = __reduce_max_sync(0xffffffffu, __float_as_uint(mx[m]));  // |x| >= 0: bits order as floats
            if (lane == 0) red[warp * 8 + m] = r;
        }
    }
    __syncthreads();
    if (tid < 8) {
        uint32_t r = 0;
        for (int w = 0; w < W; ++w) r = max(r, red[w * 8 + tid]);
        const float v = __uint_as_float(r);
        int e = 0, bad = 0;
        if (!(v <= 3.0e38f)) {
            bad = 1;  // inf or NaN somewhere in the row: its outputs become NaN
        } else if (v > 0.0f) {
            int e2;
            frexpf(v, &e2);  // v < 2^e2
            e = 22 - e2;     // max |x| * 2^e in [2^21, 2^22)
            e = e < -120 ? -120 : (e > 120 ? 120 : e);
        }
        rexp[tid] = e;
        rbad[tid] = bad;
    }
    __syncthreads();
    // Pass 2: convert.  Limb j of row m is slot s = j * M + m: row s of the
    // limb area, KS bytes; group gg's 32 bytes sit at 32-byte chunk
    // gg ^ (s & 7), and inside it, 8 bytes per word q of the group: the four
    // even k (8q, 8q+2, 8q+4, 8q+6) and then the four odd k, the order the
    // weight registers use.
    const uint32_t lbase = base + L.l_off;
    for (int ch = tid; ch < nch; ch += nthreads) {
        const int m = ch / cpr, c = ch - m * cpr;
        const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(m) * K + k0 + 8 * c);
        const float4 a = src[0], b = src[1];
        const float sc = exp2i(rexp[m]);
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        uint32_t r0[8], r1[8], r2[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            // round x * 2^e to an integer R (|R| <= 2^22) by the magic-number add
            const int R = __float_as_int(__fmaf_rn(v[i], sc, kMagic)) - kMagicBits;
            const int R1 = (R + 128) >> 8;   // R = 256 R1 + l,  l in [-128, 127]
            const int R2 = (R1 + 128) >> 8;  // R1 = 256 R2 + m
            r0[i] = static_cast<uint32_t>(R2);  // high limb (|R2| <= 64)
            r1[i] = static_cast<uint32_t>(R1);  // byte 0 = middle limb
            r2[i] = static_cast<uint32_t>(R);   // byte 0 = low limb
        }
        const int gg = c >> 2, q = c & 3;
        const uint32_t* limbs[3] = {r0, r1, r2};
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            const int s = j * M + m;
            const uint32_t* r = limbs[j];
            const uint32_t even = pack_bytes(r[0], r[2], r[4], r[6]);
            const uint32_t odd = pack_bytes(r[1], r[3], r[5], r[7]);
            sts64(lbase + s * L.ks + ((gg ^ (s & 7)) << 5) + q * 8, even, odd);
        }
    }
    // padding slots (3M .. 8 NB - 1) are zero
    for (int idx = tid; idx < (L.slots - 3 * M) * (L.ks / 8); idx += nthreads) {
        const int s = 3 * M + idx / (L.ks / 8), o = idx % (L.ks / 8);
        sts64(lbase + s * L.ks + o * 8, 0u, 0u);
    }
    __syncthreads();

    // ------------------------------------------------------------ compute --
    const int g = lane >> 2, q = lane & 3;
    float acc[NB][4];
#pragma unroll
    for (int t = 0; t < NB; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
    const int tl = warp % T, part = warp / T;
    bool ok = part < P;
    if (stall_test)  // phase 0 of box 0's barrier completes; phase 1 is never armed
        ok = mbar_wait(wfull(0), 0u, abort_flag, status, kStatusTimeoutGemv) &&
             mbar_wait(wfull(0), 1u, abort_flag, status, kStatusTimeoutGemv) && ok;
    const int gbeg = part * L.gs / P, gend = (part + 1) * L.gs / P;
    const uint32_t ra = static_cast<uint32_t>(tl * 16 + g);  // weight rows (columns) g and g + 8 of the tile
    const uint32_t wrow_a = base + L.w_off + ra * 128 + q * 4;
    const uint32_t srow_a = base + L.s_off + ra * 128;
    const uint32_t sw = static_cast<uint32_t>(g & 7);        // swizzle key of rows ra and ra + 8
    int have_box = -1, have_sbox = -1;
#pragma unroll 2
    for (int gg = gbeg; gg < gend && ok; ++gg) {
        const int b = gg >> 3, sb = gg / kIScaleBoxG;
        if (b != have_box) {
            if (!mbar_wait(wfull(b), 0u, abort_flag, status, kStatusTimeoutGemv)) { ok = false; break; }
            have_box = b;
        }
        if (sb != have_sbox) {
            if (!mbar_wait(sfull(sb), 0u, abort_flag, status, kStatusTimeoutGemv)) { ok = false; break; }
            have_sbox = sb;
        }
        const uint32_t wchunk = ((static_cast<uint32_t>(gg & 7) ^ sw) << 4);
        const uint32_t wa = lds32(wrow_a + b * L.rows * 128 + wchunk);
        const uint32_t wb = lds32(wrow_a + b * L.rows * 128 + 8 * 128 + wchunk);
        const uint32_t soff = sb * L.rows * 128 + ((static_cast<uint32_t>((gg & 31) >> 2) ^ sw) << 4) + (gg & 3) * 4;
        const float sa = ldsf(srow_a + soff);
        const float sbv = ldsf(srow_a + 8 * 128 + soff);
        // 16 v as signed bytes: even nibbles moved up, odd nibbles in place
        const uint32_t a0 = (wa << 4) & 0xF0F0F0F0u, a2 = wa & 0xF0F0F0F0u;
        const uint32_t a1 = (wb << 4) & 0xF0F0F0F0u, a3 = wb & 0xF0F0F0F0u;
#pragma unroll
        for (int t = 0; t < NB; ++t) {
            const int s = t * 8 + g;  // limb slot of this thread's B fragment (s & 7 == g)
            const uint2 bv = lds64(lbase + s * L.ks + ((static_cast<uint32_t>(gg) ^ sw) << 5) + q * 8);
            int d[4] = {kMagicBits, kMagicBits, kMagicBits, kMagicBits};
            imma_16832(d, a0, a1, a2, a3, bv.x, bv.y);
            acc[t][0] = fmaf(sa, __int_as_float(d[0]) - kMagic, acc[t][0]);
            acc[t][1] = fmaf(sa, __int_as_float(d[1]) - kMagic, acc[t][1]);
            acc[t][2] = fmaf(sbv, __int_as_float(d[2]) - kMagic, acc[t][2]);
            acc[t][3] = fmaf(sbv, __int_as_float(d[3]) - kMagic, acc[t][3]);
        }
    }

    // ------------------------------------------------------------- reduce --
    __syncthreads();  // every warp is done with the weights: their region takes the partials
    float* partv = reinterpret_cast<float*>(smem + L.part_off);  // [P][T][slots][16]
    if (part < P) {
#pragma unroll
        for (int t = 0; t < NB; ++t)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int s = t * 8 + 2 * q + j;
                float* dst = partv + ((part * T + tl) * L.slots + s) * 16;
                dst[g] = acc[t][j];
                dst[g + 8] = acc[t][2 + j];
            }
    }
    __syncthreads();
    float* cpart = reinterpret_cast<float*>(smem + L.cpart_off);  // [M][rows]: this K slice's sums
    for (int idx = tid; idx < M * L.rows; idx += nthreads) {
        const int m = idx / L.rows, r = idx - m * L.rows;
        const int tt = r >> 4, c = r & 15;
        float limb[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            float v = 0.0f;
            for (int pp = 0; pp < P; ++pp) v += partv[((pp * T + tt) * L.slots + j * M + m) * 16 + c];
            limb[j] = v;
        }
        // y = (65536 h + 256 m + l) / 16 * 2^-e  (the weights entered as 16 v)
        const float v = fmaf(limb[0], 65536.0f, fmaf(limb[1], 256.0f, limb[2]));
        cpart[idx] = rbad[m] ? __int_as_float(0x7fc00000) : v * exp2i(-rexp[m] - 4);
    }
    if (S > 1) {
        cluster_sync_all();
    } else {
        __syncthreads();
    }
    cg::cluster_group cluster = cg::this_cluster();
    // CTA crank stores columns r = crank, crank + S, ... of the cluster's block
    for (int idx = tid; idx < M * L.rows; idx += nthreads) {
        const int m = idx / L.rows, r = idx - m * L.rows;
        if (r % S != crank || r >= ncols) continue;
        float sum = 0.0f;
        if (S > 1) {
            for (int qq = 0; qq < S; ++qq) sum += cluster.map_shared_rank(cpart, qq)[idx];
        } else {
            sum = cpart[idx];
        }
        const int n = n0 + r;
        if (lora_b != nullptr) {
            float dl = 0.0f;
            for (int jr = 0; jr < rank; ++jr) dl = fmaf(lora_t[m * rank + jr], lora_b[static_cast<size_t>(jr) * N + n], dl);
            sum = fmaf(lora_scale, dl, sum);
        }
        y[static_cast<size_t>(m) * N + n] = sum;
    }
    if (S > 1) cluster_sync_all();  // peers may still read this CTA's partial sums

    if (tid == 0 && *abort_flag) {
        // copies already issued land before the CTA's shared memory is released
        for (int b = 0; b < L.nbox + L.nsbox; ++b) mbar_drain(bar + 8u * b, 0u);
    }
}

template <int NB>
int launch_imma_nb(const GemvImmaArgs& a, cudaStream_t stream) {
    const ImmaLayout L = imma_layout(a.M, a.K, a.cluster_k, a.tiles_per_cta, a.kparts);
    auto kern = q4_gemv_imma_kernel<NB>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.bytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(a.clusters * a.cluster_k));
    cfg.blockDim = dim3(static_cast<unsigned>(32 * a.tiles_per_cta * a.kparts));
    cfg.dynamicSmemBytes = static_cast<size_t>(L.bytes);
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
    e = cudaLaunchKernelEx(&cfg, kern, a.tmap_w, a.tmap_s, a.x, a.y, a.M, a.N, a.K, a.tiles_per_cta, a.kparts,
                           a.tiles_total, a.clusters, a.lora_t, a.lora_b, a.rank, a.lora_scale, a.status);
    return static_cast<int>(e);
}

}  // namespace

int gemv_imma_set_wait_test(unsigned long long limit_ns, int stall) {
    cudaError_t e = cudaMemcpyToSymbol(g_wait_limit_ns, &limit_ns, sizeof(limit_ns));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_imma_stall_test, &stall, sizeof(stall));
    return static_cast<int>(e);
}

size_t gemv_imma_smem_bytes(int M, int K, int S, int T, int P) {
    return static_cast<size_t>(imma_layout(M, K, S, T, P).bytes);
}

// Geometry: K split over a cluster of S CTAs (slices of whole 1024-k scale
// boxes), N in 16-column tiles, T tiles per CTA (at most 7, and at most what
// keeps the CTA within ~110 KB of shared memory so two share an SM), P =
// floor(16 / T) parts of each slice's groups per tile (one warp each).  With
// at most one CTA per SM the clusters share the tiles evenly; a matrix whose
// tiles do not fit one CTA per SM takes more clusters, in waves.  S (and the
// cluster count) minimise waves * T * K / S, the work of the busiest SM, ties
// to the smaller S.  Returns false when the shape does not suit the kernel.
bool gemv_imma_geometry(int sm_count, int M, int N, int K, int* S_out, int* clusters_out, int* T_out, int* P_out) {
    if (M < 1 || M > 8 || N < 1 || K <= 0 || K % 1024 != 0 || sm_count < 1) return false;
    constexpr size_t kSmemCap = 110 * 1024;
    const int tiles = (N + 15) / 16;
    long long best = -1;
    int bS = 0, bC = 0, bT = 0;
    for (int S = 1; S <= 4; S *= 2) {
        if (K % (1024 * S) != 0) continue;
        int tfit = 0;
        for (int T = 1; T <= kIMaxTiles; ++T)
            if (gemv_imma_smem_bytes(M, K, S, T, kIMaxWarps / T) <= kSmemCap) tfit = T;
        if (tfit == 0) continue;
        int C = sm_count / S;
        if (C < 1) C = 1;
        if (C > tiles) C = tiles;
        int T = (tiles + C - 1) / C;
        if (T > tfit) {  // more clusters than one per SM: waves
            T = tfit;
            C = (tiles + T - 1) / T;
        }
        const long long waves = (static_cast<long long>(C) * S + sm_count - 1) / sm_count;
        const long long work = waves * T * (K / S);
        if (best < 0 || work < best) {
            best = work;
            bS = S;
            bC = C;
            bT = T;
        }
    }
    if (best < 0) return false;
    *S_out = bS;
    *clusters_out = bC;
    *T_out = bT;
    *P_out = kIMaxWarps / bT;
    return true;
}

int launch_gemv_imma(const GemvImmaArgs& a, cudaStream_t stream) {
    if (a.M < 1 || a.M > 8 || a.K % (1024 * a.cluster_k) != 0 || a.tiles_per_cta < 1 ||
        a.tiles_per_cta > kIMaxTiles || a.kparts < 1 || a.tiles_per_cta * a.kparts > kIMaxWarps ||
        a.clusters < 1 || static_cast<long long>(a.clusters) * a.tiles_per_cta < a.tiles_total)
        return static_cast<int>(cudaErrorInvalidValue);
    switch (imma_nb(a.M)) {
        case 1: return launch_imma_nb<1>(a, stream);
        case 2: return launch_imma_nb<2>(a, stream);
        default: return launch_imma_nb<3>(a, stream);
    }
}

}  // namespace q4
