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
#include <cstdlib>

#include "common.cuh"
#include "q4_dequant.cuh"
#include "q4_kernels.h"

namespace cg = cooperative_groups;

namespace q4 {

namespace {

constexpr int kIBoxK = 256;        // k per weight box: one 128-byte row (32 words) per column
constexpr int kIScaleBoxG = 32;    // scale groups per scale box: one 128-byte row per column
constexpr int kIMaxWarps = 14;   // 448 threads: two CTAs per SM at up to 72 registers
constexpr int kIMaxTiles = 7;      // 16-column tiles per CTA (shared-memory budget)
constexpr float kMagic = 12582912.0f;          // 1.5 * 2^23
constexpr int kMagicBits = 0x4B400000;

// Test hook (gemv_imma_set_wait_test): when set, warp 0 of every CTA also
// waits for a second phase of its first weight barrier, which nothing arms,
// so that bounded wait runs out and the timeout path runs.
static __device__ int g_imma_stall_test = 0;

struct ImmaLayout {
    int ks, gs, nbox, nsbox, rows, slots, rps;
    int w_off, s_off, l_off, recv_off, red_off, bar_off, misc_off, bytes;
    int part_off;  // aliases the weight region once every warp is done with it
};

__host__ __device__ inline int imma_nb(int M) { return (3 * M + 7) / 8; }

__host__ __device__ inline ImmaLayout imma_layout(int M, int K, int S, int T, int P) {
    ImmaLayout L;
    L.ks = K / S;
    L.gs = L.ks / 32;
    L.nbox = L.ks / kIBoxK;
    L.nsbox = L.gs / kIScaleBoxG;
    L.rows = 16 * T;
    L.rps = (L.rows + S - 1) / S;  // columns each CTA of the cluster stores
    L.slots = 8 * imma_nb(M);
    L.w_off = 0;
    const int w_bytes = L.nbox * L.rows * 128;
    const int part_bytes = P * T * L.slots * 16 * 4;
    L.part_off = 0;
    const int region = w_bytes > part_bytes ? w_bytes : part_bytes;
    L.s_off = (region + 1023) / 1024 * 1024;                   // 128B-swizzled boxes: 1024-aligned
    L.l_off = L.s_off + L.nsbox * L.rows * 128;                // X slice [M][ks] fp32 by TMA, then (in place)
    const int xl = M * L.ks * 4 > L.slots * L.ks ? M * L.ks * 4 : L.slots * L.ks;  // the limb rows [slots][ks]
    L.recv_off = L.l_off + xl;                                 // [S][M][rps] fp32: the cluster's K-slice sums
    L.red_off = L.recv_off + S * M * L.rps * 4;                // row maxima [warps][8] u32, exps [8], bad [8]
    L.bar_off = (L.red_off + (kIMaxWarps * 8 + 16) * 4 + 7) / 8 * 8;
    L.misc_off = L.bar_off + (L.nbox + L.nsbox + 2) * 8;       // abort flag
    L.bytes = L.misc_off + 16;
    return L;
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
// Not volatile: a pure function of its operands, which the compiler may
// schedule (several groups' MMAs in flight at once).
__device__ __forceinline__ void imma_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// fp32 store into the shared memory of a CTA of the cluster (address from mapa).
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
// Arrive, with release semantics at cluster scope, on an mbarrier of a CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_release_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Bounded wait, with acquire semantics at cluster scope, for phase `parity` of a local mbarrier.
__device__ __forceinline__ bool mbar_wait_acquire_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                          int* status, int code) {
    const unsigned long long t0 = globaltimer_ns();
    const unsigned long long limit = *static_cast<volatile unsigned long long*>(&g_wait_limit_ns);
#pragma unroll 1
    while (true) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
        if (globaltimer_ns() - t0 > limit) {
            *abort_flag = 1;
            if (status) atomicCAS(status, 0, code);
            return false;
        }
    }
}

// Four bytes b0..b3 (byte 0 of each argument) into one word.
__device__ __forceinline__ uint32_t pack_bytes(uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3) {
    return __byte_perm(__byte_perm(b0, b1, 0x0040u), __byte_perm(b2, b3, 0x0040u), 0x5410u);
}

template <int NB>
__global__ void __launch_bounds__(kIMaxWarps * 32, 2)
    q4_gemv_imma_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_s,
                        const __grid_constant__ CUtensorMap tmap_x, float* __restrict__ y, int M, int N, int K, int T,
                        int P,
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
    const uint32_t recv_full = bar + 8u * (L.nbox + L.nsbox);  // one arrival per CTA of the cluster
    const uint32_t xfull = bar + 8u * (L.nbox + L.nsbox + 1);  // the X slice
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off);
    uint32_t* red = reinterpret_cast<uint32_t*>(smem + L.red_off);  // [kIMaxWarps][8] row-max bits
    int* rexp = reinterpret_cast<int*>(red + kIMaxWarps * 8);        // [8] row exponents
    int* rbad = rexp + 8;                                            // [8] row holds a non-finite x

    if (tid == 0) {
        for (int b = 0; b < L.nbox + L.nsbox; ++b) mbar_init(bar + 8u * b, 1);
        mbar_init(recv_full, static_cast<uint32_t>(S));
        mbar_init(xfull, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    __syncthreads();
    if (tid == 0) {
        // weights and scales do not depend on the previous launch
        tma_prefetch_desc(&tmap_w);
        tma_prefetch_desc(&tmap_s);
        tma_prefetch_desc(&tmap_x);
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
    // every CTA's receive barrier is initialised before any peer arrives on it
    // (this overlaps the previous launch: it comes before griddepcontrol.wait)
    if (S > 1) cluster_sync_all();
    pdl_wait();  // X, T and Y may belong to the previous launch until here
    if (tid == 0) {
        // this CTA's K slice of X: rows 0..M-1, boxes of 256 k
        mbar_arrive_expect_tx(xfull, static_cast<uint32_t>(M * L.ks * 4));
        for (int b = 0; b < L.ks / kIBoxK; ++b) tma_load_2d(base + L.l_off + b * kIBoxK * 4 * M, &tmap_x, xfull, k0 + b * kIBoxK, 0);
    }

    // ---------------------------------------------- X slice -> int8 limbs --
    // The slice arrives as boxes [ks/256][M][256] fp32.  Chunk ch = (row m,
    // 8 consecutive k); a thread holds all its chunks in registers (the
    // geometry keeps them at <= kXRegChunks), so after the barrier below the
    // limbs can overwrite the slice in place.
    constexpr int kXRegChunks = 3;
    const int cpr = L.ks / 8;  // chunks per row
    const int nch = M * cpr;
    float4 xr[kXRegChunks][2];
    bool ok = mbar_wait(xfull, 0u, abort_flag, status, kStatusTimeoutGemv);
    {
        float mx[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) mx[m] = 0.0f;
#pragma unroll
        for (int i = 0; i < kXRegChunks; ++i) {
            const int ch = tid + i * nthreads;
            if (ch < nch) {
                const int m = ch / cpr, c = ch - m * cpr;
                // k = 8c of row m: box c / 32, row m, element 8 (c % 32)
                const float4* src =
                    reinterpret_cast<const float4*>(smem + L.l_off + (((c >> 5) * M + m) * kIBoxK + 8 * (c & 31)) * 4);
                const float4 a = src[0], b = src[1];
                xr[i][0] = a;
                xr[i][1] = b;
                float cm = fmaxf(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))),
                                 fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
                // fmaxf drops NaN: a non-finite row is flagged through the sum
                const float sum = a.x + a.y + a.z + a.w + b.x + b.y + b.z + b.w;
                if (!isfinite(sum) || !isfinite(cm)) cm = __int_as_float(0x7f800000);  // +inf marks the row
#pragma unroll
                for (int mm = 0; mm < 8; ++mm)
                    if (mm == m) mx[mm] = fmaxf(mx[mm], cm);
            }
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            if (m >= M) break;
            const uint32_t r = __reduce_max_sync(0xffffffffu, __float_as_uint(mx[m]));  // |x| >= 0: bits order as floats
            if (lane == 0) red[warp * 8 + m] = r;
        }
    }
    __syncthreads();
    if (tid < M) {
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
    // Limb j of row m is slot s = j * M + m: row s of the limb area, KS bytes;
    // group gg's 32 bytes sit at 32-byte chunk gg ^ (s & 7), and inside it,
    // 8 bytes per word q of the group: the four even k (8q, 8q+2, 8q+4, 8q+6)
    // and then the four odd k, the order the weight registers use.
    const uint32_t lbase = base + L.l_off;
#pragma unroll
    for (int i = 0; i < kXRegChunks; ++i) {
        const int ch = tid + i * nthreads;
        if (ch >= nch) break;
        const int m = ch / cpr, c = ch - m * cpr;
        const float4 a = xr[i][0], b = xr[i][1];
        const float sc = exp2i(rexp[m]);
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        uint32_t r0[8], r1[8], r2[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            // round x * 2^e to an integer R (|R| <= 2^22) by the magic-number add
            const int R = __float_as_int(__fmaf_rn(v[e], sc, kMagic)) - kMagicBits;
            const int R1 = (R + 128) >> 8;   // R = 256 R1 + l,  l in [-128, 127]
            const int R2 = (R1 + 128) >> 8;  // R1 = 256 R2 + m
            r0[e] = static_cast<uint32_t>(R2);  // high limb (|R2| <= 64)
            r1[e] = static_cast<uint32_t>(R1);  // byte 0 = middle limb
            r2[e] = static_cast<uint32_t>(R);   // byte 0 = low limb
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
    ok = ok && part < P;
    if (stall_test)  // phase 0 of box 0's barrier completes; phase 1 is never armed
        ok = mbar_wait(wfull(0), 0u, abort_flag, status, kStatusTimeoutGemv) &&
             mbar_wait(wfull(0), 1u, abort_flag, status, kStatusTimeoutGemv) && ok;
    const int gbeg = part * L.gs / P, gend = (part + 1) * L.gs / P;
    // this warp's weight and scale boxes, all before the loop (which then has
    // no waits, so its loads and MMAs can be scheduled freely)
    if (ok && gend > gbeg) {
        for (int b = gbeg >> 3; b <= (gend - 1) >> 3 && ok; ++b)
            ok = mbar_wait(wfull(b), 0u, abort_flag, status, kStatusTimeoutGemv);
        for (int b = gbeg / kIScaleBoxG; b <= (gend - 1) / kIScaleBoxG && ok; ++b)
            ok = mbar_wait(sfull(b), 0u, abort_flag, status, kStatusTimeoutGemv);
    }
    const uint32_t ra = static_cast<uint32_t>(tl * 16 + g);  // weight rows (columns) g and g + 8 of the tile
    const uint8_t* wrow = smem + L.w_off + ra * 128 + q * 4;
    const uint8_t* srow = smem + L.s_off + ra * 128;
    const uint8_t* lrow = smem + L.l_off + q * 8;
    const uint32_t sw = static_cast<uint32_t>(g & 7);        // swizzle key of rows ra and ra + 8
    constexpr int kBatch = 4;                                // groups whose MMAs are in flight together
    if (ok) {
#pragma unroll 1
        for (int gb = gbeg; gb < gend; gb += kBatch) {
            uint32_t a0[kBatch], a1[kBatch], a2[kBatch], a3[kBatch];
            float sa[kBatch], sbv[kBatch];
            uint2 bv[kBatch][NB];
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                const int gg = min(gb + u, gend - 1);  // past the end: a repeated group, its result unused
                const int b = gg >> 3, sb = gg / kIScaleBoxG;
                const uint32_t wchunk = ((static_cast<uint32_t>(gg & 7) ^ sw) << 4);
                const uint32_t wa = *reinterpret_cast<const uint32_t*>(wrow + b * L.rows * 128 + wchunk);
                const uint32_t wb = *reinterpret_cast<const uint32_t*>(wrow + b * L.rows * 128 + 8 * 128 + wchunk);
                const uint32_t soff =
                    sb * L.rows * 128 + ((static_cast<uint32_t>((gg & 31) >> 2) ^ sw) << 4) + (gg & 3) * 4;
                sa[u] = *reinterpret_cast<const float*>(srow + soff);
                sbv[u] = *reinterpret_cast<const float*>(srow + 8 * 128 + soff);
                // 16 v as signed bytes: even nibbles moved up, odd nibbles in place
                a0[u] = (wa << 4) & 0xF0F0F0F0u;
                a2[u] = wa & 0xF0F0F0F0u;
                a1[u] = (wb << 4) & 0xF0F0F0F0u;
                a3[u] = wb & 0xF0F0F0F0u;
#pragma unroll
                for (int t = 0; t < NB; ++t) {
                    const int s = t * 8 + g;  // limb slot of this thread's B fragment (s & 7 == g)
                    bv[u][t] = *reinterpret_cast<const uint2*>(lrow + s * L.ks + ((static_cast<uint32_t>(gg) ^ sw) << 5));
                }
            }
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                const bool live = gb + u < gend;
#pragma unroll
                for (int t = 0; t < NB; ++t) {
                    int d[4] = {kMagicBits, kMagicBits, kMagicBits, kMagicBits};
                    imma_16832(d, a0[u], a1[u], a2[u], a3[u], bv[u][t].x, bv[u][t].y);
                    const float fa = live ? sa[u] : 0.0f, fb = live ? sbv[u] : 0.0f;
                    acc[t][0] = fmaf(fa, __int_as_float(d[0]) - kMagic, acc[t][0]);
                    acc[t][1] = fmaf(fa, __int_as_float(d[1]) - kMagic, acc[t][1]);
                    acc[t][2] = fmaf(fb, __int_as_float(d[2]) - kMagic, acc[t][2]);
                    acc[t][3] = fmaf(fb, __int_as_float(d[3]) - kMagic, acc[t][3]);
                }
            }
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
    // This K slice's sum of column r of row m goes to CTA r % S of the
    // cluster (the one that stores it): receive slot [crank][m][r / S].
    const uint32_t recv_local = base + L.recv_off;
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
        const float val = rbad[m] ? __int_as_float(0x7fc00000) : v * exp2i(-rexp[m] - 4);
        const int owner = r % S;
        const uint32_t slot = recv_local + static_cast<uint32_t>(((crank * M + m) * L.rps + r / S) * 4);
        if (owner == crank) {
            *reinterpret_cast<float*>(smem + (slot - base)) = val;
        } else {
            st_cluster_f32(mapa_shared(slot, static_cast<uint32_t>(owner)), val);
        }
    }
    __syncthreads();  // every thread's stores of its sums are ordered before thread 0's release below
    if (tid == 0) {
        if (S > 1) asm volatile("fence.acq_rel.cluster;" ::: "memory");
        for (int o = 0; o < S; ++o)
            mbar_arrive_release_cluster(S > 1 ? mapa_shared(recv_full, static_cast<uint32_t>(o)) : recv_full);
    }
    // every CTA of the cluster has delivered its slice's sums for this CTA's columns
    mbar_wait_acquire_cluster(recv_full, 0u, abort_flag, status, kStatusTimeoutGemv);
    const float* recv = reinterpret_cast<const float*>(smem + L.recv_off);
    for (int idx = tid; idx < M * L.rps; idx += nthreads) {
        const int m = idx / L.rps, rr = idx - m * L.rps;
        const int r = rr * S + crank;
        if (r >= ncols) continue;
        float sum = 0.0f;
        for (int j = 0; j < S; ++j) sum += recv[(j * M + m) * L.rps + rr];  // fixed order: deterministic
        const int n = n0 + r;
        if (lora_b != nullptr) {
            float dl = 0.0f;
            for (int jr = 0; jr < rank; ++jr) dl = fmaf(lora_t[m * rank + jr], lora_b[static_cast<size_t>(jr) * N + n], dl);
            sum = fmaf(lora_scale, dl, sum);
        }
        y[static_cast<size_t>(m) * N + n] = sum;
    }

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
    e = cudaLaunchKernelEx(&cfg, kern, a.tmap_w, a.tmap_s, a.tmap_x, a.y, a.M, a.N, a.K, a.tiles_per_cta, a.kparts,
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
// floor(14 / T) parts of each slice's groups per tile (one warp each).  With
// at most one CTA per SM the clusters share the tiles evenly; a matrix whose
// tiles do not fit one CTA per SM takes more clusters, in waves.  S (and the
// cluster count) minimise waves * T * K / S, the work of the busiest SM, ties
// to the smaller S.  Returns false when the shape does not suit the kernel.
bool gemv_imma_geometry(int sm_count, int M, int N, int K, int* S_out, int* clusters_out, int* T_out, int* P_out) {
    if (M < 1 || M > 8 || N < 1 || K <= 0 || K % 1024 != 0 || sm_count < 1) return false;
    constexpr size_t kSmemCap = 110 * 1024;
    // SPACESLUG_Q4_IMMA_SPLIT=1|2|4 forces the K split (when the shape allows it)
    static const int forced = [] {
        const char* e = std::getenv("SPACESLUG_Q4_IMMA_SPLIT");
        const int v = e ? std::atoi(e) : 0;
        return (v == 1 || v == 2 || v == 4) ? v : 0;
    }();
    const int tiles = (N + 15) / 16;
    long long best = -1;
    int bS = 0, bC = 0, bT = 0;
    for (int S = 1; S <= 4; S *= 2) {
        if (K % (1024 * S) != 0 || (forced != 0 && S != forced)) continue;
        // each thread holds all its chunks of the X slice (<= 3) in registers
        int tfit = 0;
        for (int T = 1; T <= kIMaxTiles; ++T)
            if (gemv_imma_smem_bytes(M, K, S, T, kIMaxWarps / T) <= kSmemCap &&
                static_cast<long long>(M) * (K / S) / 8 <= 3LL * 32 * T * (kIMaxWarps / T))
                tfit = T;
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
    if (static_cast<long long>(a.M) * (a.K / (a.cluster_k > 0 ? a.cluster_k : 1)) / 8 >
            3LL * 32 * a.tiles_per_cta * a.kparts)
        return static_cast<int>(cudaErrorInvalidValue);  // X slice chunks must fit the threads' registers
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
