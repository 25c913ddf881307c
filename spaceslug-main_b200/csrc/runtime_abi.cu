// Host runtime behind include/runtime_abi.h: argument validation, per-device
// context (status word, stream for synchronous calls, stream-ordered scratch
// pool), TMA descriptor encoding, kernel dispatch (GEMV for M <= 8, tcgen05
// GEMM above), device-resident weight handles.
//
// Error behaviour mirrors vulkan-runtime/src/api/lora_delta_api.cpp:42-85:
// arguments are checked first (return 1), every device failure returns 2, and
// nothing throws across the ABI (catch (...) -> 2).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <memory>
#include <array>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/runtime_abi.h"
#include "q4_kernels.h"
#include "upload.h"

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};
std::atomic<int> g_operand{static_cast<int>(q4::Operand16::kF16)};
std::atomic<int> g_decode_variant{0};  // 0 auto, 1 ring GEMV, 2 tcgen05 decode, 3 whole-tile GEMV, 4 IMMA GEMV
std::atomic<int> g_gemm_variant{0};  // 0 auto, 1 single-CTA 128-row tiles, 2 CTA pair, 3 single-CTA 256-row tiles
std::once_flag g_operand_env_once;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

struct CudaError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw CudaError(std::string(what) + ": " + cudaGetErrorString(e));
}
void check_launch(int e, const char* what) {
    if (e != 0) throw CudaError(std::string(what) + ": " + cudaGetErrorString(static_cast<cudaError_t>(e)));
    g_launches.fetch_add(1, std::memory_order_relaxed);
}

// ------------------------------------------------------------ device ctx --
struct DeviceCtx {
    std::once_flag once;
    bool ok = false;
    std::atomic<bool> ready{false};  // ok, published for readers that must not initialise the context
    std::string init_error;
    int sm_count = 0;
    int* status = nullptr;  // device int, kernels record wait timeouts here
    int* status_host = nullptr;     // pinned, mapped host word the host entry points read `status` into
    int* status_host_dev = nullptr; // its device address
    int* done_host = nullptr;       // pinned, mapped word a host call's last kernel sets when it is done
    int* done_host_dev = nullptr;   // its device address
    unsigned* done_count = nullptr; // device counter of the CTAs of that kernel that have finished
    cudaStream_t stream = nullptr;  // for the synchronous host-pointer entry points
    std::mutex host_mu;             // serialises use of `stream` and `hbuf` by host entry points
    void* hbuf = nullptr;           // device staging of X and Y for spaceslug_q4_weights_run_host (grows)
    size_t hbuf_bytes = 0;
    uint64_t hbuf_gen = 0;          // bumped whenever hbuf is replaced (graphs of host calls name it)
    int max_pairs[2] = {-1, -1};    // co-resident CTA pairs of the pair GEMM, per operand type
    std::mutex pair_mu;
    cudaStream_t aux = nullptr;     // lowest-priority helper stream for work forked off a call (lazy)
    std::mutex aux_mu;              // held while a call forks onto `aux` and joins back
};

// The device's helper stream (created on first use).
cudaStream_t aux_stream(DeviceCtx& c) {
    if (c.aux == nullptr) {
        int least = 0, greatest = 0;
        check(cudaDeviceGetStreamPriorityRange(&least, &greatest), "cudaDeviceGetStreamPriorityRange");
        check(cudaStreamCreateWithPriority(&c.aux, cudaStreamNonBlocking, least), "cudaStreamCreate (aux)");
    }
    return c.aux;
}

// An event for one fork or join of a call (released when the call returns;
// destroying an event with work pending is allowed).
struct CallEvent {
    cudaEvent_t e = nullptr;
    CallEvent() { check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate"); }
    ~CallEvent() {
        if (e) cudaEventDestroy(e);
    }
    CallEvent(const CallEvent&) = delete;
    CallEvent& operator=(const CallEvent&) = delete;
};

constexpr int kMaxDevices = 64;
DeviceCtx g_ctx[kMaxDevices];

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;

EncodeTiledFn encoder() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    });
    if (!g_encode) throw CudaError("cuTensorMapEncodeTiled is unavailable");
    return g_encode;
}

DeviceCtx& ctx_for(int device) {
    if (device < 0 || device >= kMaxDevices) throw CudaError("device ordinal out of range");
    DeviceCtx& c = g_ctx[device];
    std::call_once(c.once, [&] {
        try {
            check(cudaSetDevice(device), "cudaSetDevice");
            check(cudaDeviceGetAttribute(&c.sm_count, cudaDevAttrMultiProcessorCount, device), "sm count");
            int major = 0, minor = 0;
            check(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device), "cc major");
            check(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device), "cc minor");
            if (major != 10) throw CudaError("this library is built for sm_100a (B200); device is sm_" +
                                             std::to_string(major) + std::to_string(minor));
            check(cudaMalloc(&c.status, sizeof(int)), "cudaMalloc status");
            check(cudaMemset(c.status, 0, sizeof(int)), "cudaMemset status");
            // status word at 0, completion word 64 bytes on
            check(cudaHostAlloc(reinterpret_cast<void**>(&c.status_host), 128, cudaHostAllocMapped),
                  "cudaHostAlloc status");
            check(cudaHostGetDevicePointer(reinterpret_cast<void**>(&c.status_host_dev), c.status_host, 0),
                  "cudaHostGetDevicePointer status");
            *c.status_host = 0;
            c.done_host = c.status_host + 16;
            c.done_host_dev = c.status_host_dev + 16;
            *c.done_host = 0;
            check(cudaMalloc(reinterpret_cast<void**>(&c.done_count), sizeof(unsigned)), "cudaMalloc done count");
            check(cudaMemset(c.done_count, 0, sizeof(unsigned)), "cudaMemset done count");
            check(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking), "cudaStreamCreate");
            cudaMemPool_t pool;
            check(cudaDeviceGetDefaultMemPool(&pool, device), "default mem pool");
            uint64_t keep = UINT64_MAX;
            check(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep), "pool threshold");
            c.ok = true;
            c.ready.store(true, std::memory_order_release);
        } catch (const std::exception& e) {
            c.init_error = e.what();
        }
    });
    if (!c.ok) throw CudaError(c.init_error.empty() ? "device init failed" : c.init_error);
    return c;
}

int current_device() {
    int d = 0;
    check(cudaGetDevice(&d), "cudaGetDevice");
    return d;
}

// Decode variant; SPACESLUG_Q4_DECODE=auto|gemv|mma|tile sets its initial value.
std::atomic<int>& decode_variant_init() {
    static std::once_flag once;
    std::call_once(once, [] {
        const char* e = std::getenv("SPACESLUG_Q4_DECODE");
        const char* names[5] = {"auto", "gemv", "mma", "tile", "imma"};
        for (int i = 0; e && i < 5; ++i)
            if (std::strcmp(e, names[i]) == 0) g_decode_variant.store(i);
    });
    return g_decode_variant;
}

q4::Operand16 operand_type() {
    std::call_once(g_operand_env_once, [] {
        const char* e = std::getenv("SPACESLUG_Q4_OPERAND");
        if (e && std::strcmp(e, "bf16") == 0) g_operand.store(static_cast<int>(q4::Operand16::kBF16));
        if (e && std::strcmp(e, "f16") == 0) g_operand.store(static_cast<int>(q4::Operand16::kF16));
    });
    return static_cast<q4::Operand16>(g_operand.load());
}

// Stream-ordered scratch buffer released on the same stream at scope exit.
struct Scratch {
    void* p = nullptr;
    cudaStream_t s = nullptr;
    Scratch(size_t bytes, cudaStream_t stream) : s(stream) {
        if (bytes) check(cudaMallocAsync(&p, bytes, stream), "cudaMallocAsync");
    }
    ~Scratch() {
        if (p) cudaFreeAsync(p, s);
    }
    Scratch(const Scratch&) = delete;
    Scratch& operator=(const Scratch&) = delete;
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Argument check shared by all GEMM entry points (reference convention:
// before any device work, return 1).
const char* shape_error(const void* x, const void* packed, const void* scales, const void* y, uint32_t m, uint32_t n,
                        uint32_t k, uint32_t rank, const void* la, const void* lb, float alpha) {
    if (!x || !packed || !scales || !y) return "null pointer";
    if (m == 0 || n == 0 || k == 0) return "zero dimension";
    if (k % 32u) return "k must be a multiple of 32 (the scale group size)";
    if (m > (1u << 30) || n > (1u << 30) || k > (1u << 30)) return "dimension too large";
    if (rank > 64) return "LoRA rank must be <= 64";
    if (rank > 0 && (!la || !lb)) return "LoRA rank > 0 needs both A and B";
    if (rank > 0 && !std::isfinite(alpha)) return "LoRA alpha must be finite";
    return nullptr;
}

// --------------------------------------------------------------- dispatch --
// Tensor maps of a weight handle's decode launches, encoded once per
// geometry instead of once per call: the integer-MMA GEMV's weight and scale
// maps, the whole-tile GEMV's, and the tile GEMV's last X map (the host-pointer
// calls stage X in a per-device buffer, so its address repeats call after call).
struct DecodeMapCache {
    std::mutex mu;
    int S = 0, T = 0;  // geometry the integer-MMA maps were encoded for (0: none yet)
    CUtensorMap w{}, s{};
    uint32_t tile_rows = 0;  // box rows the whole-tile maps were encoded for (0: none yet)
    CUtensorMap tile_w{}, tile_s{};
    const void* x_ptr = nullptr;  // the X the cached X map describes, with its M and K split
    int x_m = 0, x_split = 0;
    CUtensorMap tile_x{};
};

struct Problem {
    const float* x;
    const uint32_t* packed;
    const float* scales;
    const int* col_exp;  // precomputed per-column exponents (handles) or nullptr
    const float* lora_a;
    const float* lora_b;
    int rank;
    float alpha;
    float* y;
    int M, N, K;
    long long ld_y = 0;  // row pitch of Y in floats (0: N)
    int sm_budget = 0;   // SMs the GEMM may occupy (0: all)
    const q4::PeerPtrs* peers = nullptr;  // Y also stored to these peers' Y (same offsets and pitch)
    int npeers = 0;
    DecodeMapCache* maps = nullptr;       // a weight handle's cached decode tensor maps, or nullptr
};

// GEMV launch geometry.  K is split over a cluster of S CTAs (S | G, slice
// of GS = G/S <= 32 groups so one lane owns one group); one CTA per SM; the
// column range per cluster is a multiple of the 16-column chunk.  Returns
// false when the GEMV cannot take the shape (the caller uses the GEMM).
struct GemvGeom {
    int S = 0, clusters = 0, cols = 0;
};
std::mutex g_geom_mu;
std::vector<std::pair<std::array<int, 4>, int>> g_geom_cache;  // (M, K, S, cols) -> max clusters

int cached_max_clusters(int M, int K, int S, int cols) {
    std::array<int, 4> key{M, K, S, cols};
    {
        std::lock_guard<std::mutex> lk(g_geom_mu);
        for (auto& e : g_geom_cache)
            if (e.first == key) return e.second;
    }
    const int v = q4::gemv_max_active_clusters(M, K, S, cols);
    std::lock_guard<std::mutex> lk(g_geom_mu);
    g_geom_cache.emplace_back(key, v);
    return v;
}

bool choose_gemv(const DeviceCtx& c, int M, int N, int K, GemvGeom& out) {
    const int G = K / 32;
    int S = 0;
    for (int cand = 1; cand <= 8; cand *= 2) {
        if (G % cand) continue;
        const int gs = G / cand;
        if (gs > 32) continue;
        S = cand;
        break;
    }
    if (S == 0) return false;
    const int cc = q4::gemv_chunk_columns();
    const int target = std::max(1, c.sm_count / S);
    int clusters = std::max(1, std::min(target, (N + cc - 1) / cc));
    int cols = (N + clusters - 1) / clusters;
    cols = (cols + cc - 1) / cc * cc;
    if (q4::gemv_smem_bytes(M, K, S, cols) > 200 * 1024) return false;
    const int resident = cached_max_clusters(M, K, S, cols);
    if (resident <= 0) return false;
    if (resident < clusters) {
        clusters = resident;
        cols = (N + clusters - 1) / clusters;
        cols = (cols + cc - 1) / cc * cc;
    }
    out.S = S;
    out.cols = cols;
    out.clusters = (N + cols - 1) / cols;
    return true;
}

// K split (cluster size) of the whole-tile GEMV: the smallest that fits in
// shared memory; SPACESLUG_Q4_TILE_SPLIT overrides (1, 2, 4 or 8).
int tile_split(int M, int K) {
    static const int forced = [] {
        const char* e = std::getenv("SPACESLUG_Q4_TILE_SPLIT");
        const int s = e ? std::atoi(e) : 0;
        return (s == 1 || s == 2 || s == 4 || s == 8) ? s : 0;
    }();
    if (forced > 0) return q4::gemv_tile_supported(M, K, forced) ? forced : 0;
    for (int S = 1; S <= 8; S *= 2)
        if (q4::gemv_tile_supported(M, K, S)) return S;
    return 0;
}

void encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encoder()(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")");
}

// Co-resident clusters of the pair SGEMM on the current device (cached).
int sgemm_pairs_on_device() {
    static std::atomic<int> cache[64];
    static std::atomic<bool> init[64];
    int dev = 0;
    check(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= 64) return q4::sgemm_pair_max_active();
    if (!init[dev].load(std::memory_order_acquire)) {
        cache[dev].store(q4::sgemm_pair_max_active(), std::memory_order_relaxed);
        init[dev].store(true, std::memory_order_release);
    }
    return cache[dev].load(std::memory_order_relaxed);
}

// Pair tiles (256 x 256, MMA-bound, ~1548 cycles per 32-k stage) or single
// tiles (128 x bn, shared-memory-bound, ~1250 cycles per stage at bn = 128):
// the one whose waves of stages take less time.
bool sgemm_use_pair(int m, int n, int sm_count, int pairs) {
    if (m < 256 || n < 256 || pairs < 1) return false;
    const long long single_waves = (static_cast<long long>((m + 127) / 128) * ((n + 127) / 128) + sm_count - 1) / sm_count;
    const long long pair_waves = (static_cast<long long>(q4::sgemm_pair_tiles(m, n)) + pairs - 1) / pairs;
    return pair_waves * 1548 < single_waves * 1250;
}

// fp32 GEMM C[m x n] (row pitch ldc) = alpha * op(A) op(B) on the tcgen05
// tensor cores (3xTF32, sgemm_tc.cu).  op(A) is [m x k]: A row-major [m][k]
// with row pitch lda, or with trans_a A given as [k][m]; op(B) is [k x n]: B
// row-major [k][n] with row pitch ldb, or with trans_b B given as [n][k].  The
// operands' TF32 hi / lo planes live in stream-ordered scratch.
void run_sgemm(const float* a, long long lda, bool trans_a, const float* b, long long ldb, bool trans_b, float* cm,
               long long ldc, int m, int n, int k, float alpha, int* status, cudaStream_t stream) {
    int dev = 0, sms = 0;
    check(cudaGetDevice(&dev), "cudaGetDevice");
    check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
    const int pairs = m >= 256 && n >= 256 ? sgemm_pairs_on_device() : 0;
    const bool pair = sgemm_use_pair(m, n, sms, pairs);
    // Planes padded to whole TMA boxes (zeros): k to a multiple of 32, the rows
    // to whole tiles (128 rows of A and bn of B, or 256 of both for pairs), so
    // every box lies inside its plane.
    const int bn = q4::sgemm_tc_bn(n);
    const long long ldk = (static_cast<long long>(k) + 31) / 32 * 32;
    const int mt = pair ? 256 : 128, nt = pair ? 256 : bn;
    const int mr = (m + mt - 1) / mt * mt, nr = (n + nt - 1) / nt * nt;
    Scratch pa(static_cast<size_t>(2) * mr * ldk * sizeof(float), stream);
    Scratch pb(static_cast<size_t>(2) * nr * ldk * sizeof(float), stream);
    float* ahi = static_cast<float*>(pa.p);
    float* alo = ahi + static_cast<size_t>(mr) * ldk;
    float* bhi = static_cast<float*>(pb.p);
    float* blo = bhi + static_cast<size_t>(nr) * ldk;
    if (trans_a)
        check_launch(q4::launch_split_planes(a, k, m, lda, true, ahi, alo, mr, ldk, stream), "split A");
    else
        check_launch(q4::launch_split_planes(a, m, k, lda, false, ahi, alo, mr, ldk, stream), "split A");
    if (trans_b)
        check_launch(q4::launch_split_planes(b, n, k, ldb, false, bhi, blo, nr, ldk, stream), "split B");
    else
        check_launch(q4::launch_split_planes(b, k, n, ldb, true, bhi, blo, nr, ldk, stream), "split B");
    q4::SgemmTcArgs g{};
    g.bn = bn;
    const uint64_t rb = static_cast<uint64_t>(ldk) * 4;
    const uint64_t kk = static_cast<uint64_t>(ldk);
    encode_2d(&g.tm_ahi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ahi, kk, mr, rb, 32, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    encode_2d(&g.tm_alo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, alo, kk, mr, rb, 32, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    const uint32_t b_box = pair ? 128u : static_cast<uint32_t>(bn);  // a pair CTA loads 128 rows of B
    encode_2d(&g.tm_bhi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, bhi, kk, nr, rb, 32, b_box, CU_TENSOR_MAP_SWIZZLE_128B);
    encode_2d(&g.tm_blo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, blo, kk, nr, rb, 32, b_box, CU_TENSOR_MAP_SWIZZLE_128B);
    g.c = cm;
    g.M = m; g.N = n; g.K = k;
    g.ldc = ldc;
    g.alpha = alpha;
    g.status = status;
    if (pair)
        check_launch(q4::launch_sgemm_pair(g, pairs, stream), "sgemm (tcgen05 pairs) launch");
    else
        check_launch(q4::launch_sgemm_tc(g, stream), "sgemm (tcgen05) launch");
}

// The LoRA backward takes the tensor-core passes of lora_tc.cu when the
// operands suit their TMA maps: X [M][K] and dY [M][N] 16-byte aligned with
// 16-byte row strides (K, N multiples of 4), every box inside its tensor
// (M >= 128 rows for the 128-row boxes, K, N >= 32), rank <= 64.
// SPACESLUG_LORA_BACKWARD=fma keeps the CUDA-core kernels of lora_train.cu.
bool lora_backward_tc_suits(const q4::LoraBackwardArgs& g) {
    static const bool fma_only = [] {
        const char* e = std::getenv("SPACESLUG_LORA_BACKWARD");
        return e && std::string(e) == "fma";
    }();
    return !fma_only && g.M >= 128 && g.K >= 32 && g.N >= 32 && g.K % 4 == 0 && g.N % 4 == 0 && g.rank >= 1 &&
           g.rank <= 64 && aligned16(g.x) && aligned16(g.dy);
}

// T = X A, G = dY B^T, dB = s T^T dY, dA = s X^T G as tcgen05 passes, in
// five launches: the A^T and B planes; the T and G passes (X and dY rows,
// one launch); their split sums as T^T and G^T planes; the dB and dA passes
// (dY and X transposed, one launch); their split sums scaled into dB and dA.
// The narrow operands enter the passes as stacked TF32 hi / lo planes
// [2 rp][L].
void run_lora_backward_tc(const q4::LoraBackwardArgs& g, int sm_count, int* status, cudaStream_t s) {
    const int M = g.M, K = g.K, N = g.N, r = g.rank, rp = q4::lora_tc_rp(r);
    auto round4 = [](int v) { return (static_cast<long long>(v) + 3) / 4 * 4; };
    const long long Kp = round4(K), Np = round4(N), Mp = round4(M);
    int s1[2], s2[2];
    {
        const int R1[2] = {M, M}, L1[2] = {K, N}, R2[2] = {N, K}, L2[2] = {M, M};
        q4::lora_tc_plan(2, R1, L1, sm_count, s1);
        q4::lora_tc_plan(2, R2, L2, sm_count, s2);
    }
    const long long partA = static_cast<long long>(s1[0]) * M * rp, partB = static_cast<long long>(s1[1]) * M * rp;
    const long long partC = static_cast<long long>(s2[0]) * N * rp, partD = static_cast<long long>(s2[1]) * K * rp;
    const long long part = std::max(partA + partB, partC + partD);
    const long long two = 2ll * rp;
    Scratch sc(static_cast<size_t>(two * (Kp + Np + 2 * Mp) + part) * sizeof(float), s);
    float* astk = static_cast<float*>(sc.p);
    float* bstk = astk + two * Kp;
    float* tstk = bstk + two * Np;
    float* gstk = tstk + two * Mp;
    float* part0 = gstk + two * Mp;
    const auto F32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
    const uint32_t brows = static_cast<uint32_t>(two);
    auto problem = [&](q4::LoraTcProblem& q, const float* a, uint64_t a_inner, uint64_t a_outer, bool mn_major,
                       const float* bplane, int R, int L, int splits, float* partial) {
        // K-major: 32 l x 128 rows of D, 128-byte swizzle; MN-major: 128 rows of D (contiguous) x 32 l, unswizzled
        encode_2d(&q.tm_a, F32, a, a_inner, a_outer, a_inner * 4, mn_major ? 128 : 32, mn_major ? 32 : 128,
                  mn_major ? CU_TENSOR_MAP_SWIZZLE_NONE : SW);
        encode_2d(&q.tm_b, F32, bplane, static_cast<uint64_t>(L), two, static_cast<uint64_t>(round4(L)) * 4, 32,
                  brows, SW);
        q.partial = partial;
        q.R = R;
        q.L = L;
        q.splits = splits;
    };
    q4::LoraTcFinalize f[2];
    // A^T planes (A is [K][r]: its rows are the planes' columns) and B planes
    f[0] = {g.lora_a, 1, K, r, r, 0, 1.0f, astk, Kp};
    f[1] = {g.lora_b, 1, N, N, r, 3, 1.0f, bstk, Np};
    check_launch(q4::launch_lora_tc_finalize(f, 2, rp, s), "lora A / B planes");
    q4::LoraTcPass p{};
    p.count = 2;
    p.rp = rp;
    p.sm_count = sm_count;
    p.status = status;
    // T = X A (rows m of X, B operand A^T) and G = dY B^T (rows m of dY, B operand B)
    float* partT = part0;
    float* partG = part0 + partA;
    problem(p.prob[0], g.x, K, M, false, astk, M, K, s1[0], partT);
    problem(p.prob[1], g.dy, N, M, false, bstk, M, N, s1[1], partG);
    p.mn_major = 0;
    check_launch(q4::launch_lora_tc_pass(p, s), "lora T / G pass");
    f[0] = {partT, s1[0], M, rp, r, 0, 1.0f, tstk, Mp};
    f[1] = {partG, s1[1], M, rp, r, 0, 1.0f, gstk, Mp};
    check_launch(q4::launch_lora_tc_finalize(f, 2, rp, s), "lora T / G planes");
    // dB^T = dY^T T (rows n of dY^T, B operand T^T) and dA = X^T G (rows k of X^T, B operand G^T)
    float* partB2 = part0;
    float* partA2 = part0 + partC;
    problem(p.prob[0], g.dy, N, M, true, tstk, N, M, s2[0], partB2);
    problem(p.prob[1], g.x, K, M, true, gstk, K, M, s2[1], partA2);
    p.mn_major = 1;
    check_launch(q4::launch_lora_tc_pass(p, s), "lora dB / dA pass");
    f[0] = {partB2, s2[0], N, rp, r, 1, g.scale, g.db, N};
    f[1] = {partA2, s2[1], K, rp, r, 2, g.scale, g.da, r};
    check_launch(q4::launch_lora_tc_finalize(f, 2, rp, s), "lora dB / dA");
}

// Co-resident CTA pairs of the pair kernel for operand type `op` (cached).
int pair_capacity(DeviceCtx& c, q4::Operand16 op) {
    std::lock_guard<std::mutex> lk(c.pair_mu);
    int& mp = c.max_pairs[static_cast<int>(op)];
    if (mp < 0) mp = q4::gemm_pair_max_active(op);
    return mp;
}

// K split of the pair kernel: 2 when the tiles fill at most half of the
// co-resident pairs (two K halves per tile then fit one wave) and each half
// is whole 128-k stages of a long enough K.
int pair_ksplit(const Problem& p, int pairs) {
    const int tiles = q4::gemm_pair_tiles(p.M, p.N);
    return (p.K % 256 == 0 && p.K >= 1024 && 2 * tiles <= pairs) ? 2 : 1;
}

// The GEMM takes the CTA-pair kernel (256 x 256 tiles, half the operand bytes
// per FLOP, the dequantised weights in tensor memory, a deeper pipeline per
// SM) whenever the shape suits its TMA maps: scales loaded with row stride
// K/8 bytes (K % 128 == 0), Y stored with row stride 4 ld bytes (N % 4 == 0,
// ld % 4 == 0, 16-byte aligned Y).  Measured on B200 it beats the
// single-CTA kernel also when its units do not fill the pairs (M = 256 to
// 1024 at K = N = 4096: 33 / 35 / 82 us against 50 / 52 / 115 us, the last
// with LoRA).  Its epilogue adds the LoRA term in fp32.
bool use_pair_kernel(DeviceCtx& c, const Problem& p, q4::Operand16 op, int* pairs_out) {
    const long long ld = p.ld_y ? p.ld_y : p.N;
    int pairs = pair_capacity(c, op);
    if (p.sm_budget > 0 && pairs > p.sm_budget / 2) pairs = p.sm_budget / 2;
    if (pairs_out) *pairs_out = pairs;
    const int variant = g_gemm_variant.load();
    bool shape_ok = p.K % 128 == 0 && p.N % 4 == 0 && ld % 4 == 0 && aligned16(p.y) && aligned16(p.scales);
    for (int q = 0; q < p.npeers; ++q) shape_ok = shape_ok && aligned16(p.peers->p[q]);  // 16-byte peer stores
    return p.rank <= 64 && pairs > 0 && shape_ok && (variant == 0 || variant == 2);
}

void run_problem(const Problem& p, cudaStream_t stream) {
    DeviceCtx& c = ctx_for(current_device());
    if (p.npeers > 0 && !(p.M > 8 && use_pair_kernel(c, p, operand_type(), nullptr))) {
        // Only the pair kernel pushes from its epilogue: elsewhere the product
        // is written here first and then pushed as one block.
        Problem q = p;
        q.peers = nullptr;
        q.npeers = 0;
        run_problem(q, stream);
        check_launch(q4::launch_push_rows(p.y, *p.peers, p.npeers, p.M, p.N, p.ld_y ? p.ld_y : p.N,
                                          2 * c.sm_count, stream),
                     "push_rows");
        return;
    }
    if (p.ld_y != 0 && p.ld_y != p.N && !(p.M > 8 && use_pair_kernel(c, p, operand_type(), nullptr))) {
        // Only the pair kernel (reached for M > 8) stores Y with an arbitrary
        // row pitch: elsewhere the product lands in scratch and one strided
        // copy places it.
        Scratch ys(static_cast<size_t>(p.M) * p.N * sizeof(float), stream);
        Problem q = p;
        q.y = static_cast<float*>(ys.p);
        q.ld_y = 0;
        run_problem(q, stream);
        check(cudaMemcpy2DAsync(p.y, static_cast<size_t>(p.ld_y) * 4, ys.p, static_cast<size_t>(p.N) * 4,
                                static_cast<size_t>(p.N) * 4, static_cast<size_t>(p.M), cudaMemcpyDeviceToDevice,
                                stream),
              "cudaMemcpy2DAsync (strided Y)");
        return;
    }
    Scratch t_buf(p.rank > 0 ? static_cast<size_t>(p.M) * p.rank * sizeof(float) : 0, stream);
    Scratch t_part(p.rank > 0 ? static_cast<size_t>(q4::lora_xa_chunks(p.K)) * p.M * p.rank * sizeof(float) : 0,
                   stream);
    float* lora_t = static_cast<float*>(t_buf.p);
    // The decode kernels add (alpha/r) * T * B in their epilogue from fp32 T;
    // the GEMM computes T after the X cast (it needs the row exponents).
    if (p.rank > 0 && p.M <= 8)
        check_launch(q4::launch_lora_xa(p.x, p.lora_a, lora_t, p.M, p.K, p.rank, stream,
                                        static_cast<float*>(t_part.p)),
                     "lora_xa");
    const float lscale = p.rank > 0 ? p.alpha / static_cast<float>(p.rank) : 0.0f;

    // Decode (M <= 8).  Automatic choice: the whole-tile GEMV where the shape
    // allows it, else the streamed-ring GEMV.  The integer-tensor-core GEMV
    // and the tcgen05 decode run on request only: measured in a 24-layer
    // CUDA graph at K = N = 4096 they are slower per layer at every M (the
    // integer-MMA one: 10.4 / 10.7 / 13.2 / 17.0 us at M = 1 / 2 / 4 / 8,
    // against 4.9 / 5.7 / 9.0 / 11.9 us for the whole-tile GEMV).
    const int dv = decode_variant_init().load();
    if (p.M <= 8 && dv == 4 && aligned16(p.x) && aligned16(p.packed) && aligned16(p.scales)) {
        q4::GemvImmaArgs a{};
        if (q4::gemv_imma_geometry(c.sm_count, p.M, p.N, p.K, &a.cluster_k, &a.clusters, &a.tiles_per_cta,
                                   &a.kparts)) {
            const int K = p.K, N = p.N;
            const uint32_t rows = static_cast<uint32_t>(16 * a.tiles_per_cta);
            auto encode = [&](CUtensorMap* mw, CUtensorMap* ms) {
                encode_2d(mw, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.packed, static_cast<uint64_t>(K) / 8,
                          static_cast<uint64_t>(N), static_cast<uint64_t>(K) / 2, 32, rows, CU_TENSOR_MAP_SWIZZLE_128B);
                encode_2d(ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.scales, static_cast<uint64_t>(K) / 32,
                          static_cast<uint64_t>(N), static_cast<uint64_t>(K) / 8, 32, rows, CU_TENSOR_MAP_SWIZZLE_128B);
            };
            if (p.maps != nullptr) {
                std::lock_guard<std::mutex> lk(p.maps->mu);
                if (p.maps->S != a.cluster_k || p.maps->T != a.tiles_per_cta) {
                    encode(&p.maps->w, &p.maps->s);
                    p.maps->S = a.cluster_k;
                    p.maps->T = a.tiles_per_cta;
                }
                a.tmap_w = p.maps->w;
                a.tmap_s = p.maps->s;
            } else {
                encode(&a.tmap_w, &a.tmap_s);
            }
            encode_2d(&a.tmap_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.x, static_cast<uint64_t>(K),
                      static_cast<uint64_t>(p.M), static_cast<uint64_t>(K) * 4, 256, static_cast<uint32_t>(p.M),
                      CU_TENSOR_MAP_SWIZZLE_NONE);
            a.y = p.y;
            a.M = p.M; a.N = N; a.K = K;
            a.tiles_total = (N + 15) / 16;
            a.lora_t = lora_t; a.lora_b = p.rank > 0 ? p.lora_b : nullptr; a.rank = p.rank; a.lora_scale = lscale;
            a.status = c.status;
            check_launch(q4::launch_gemv_imma(a, stream), "gemv imma launch");
            return;
        }
    }
    if (p.M <= 8 && (dv == 0 || dv == 3)) {
        const int S = tile_split(p.M, p.K);
        if (S > 0 && aligned16(p.x) && aligned16(p.packed) && aligned16(p.scales)) {
            q4::GemvTileArgs a{};
            const int K = p.K, N = p.N;
            a.col_blocks = q4::gemv_tile_col_blocks(N, c.sm_count);
            const uint32_t rows = static_cast<uint32_t>(q4::gemv_tile_box_rows(N, a.col_blocks));
            auto encode_ws = [&](CUtensorMap* mw, CUtensorMap* ms) {
                encode_2d(mw, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.packed, static_cast<uint64_t>(K) / 8,
                          static_cast<uint64_t>(N), static_cast<uint64_t>(K) / 2, 32, rows, CU_TENSOR_MAP_SWIZZLE_128B);
                encode_2d(ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.scales, static_cast<uint64_t>(K) / 32,
                          static_cast<uint64_t>(N), static_cast<uint64_t>(K) / 8,
                          static_cast<uint32_t>(q4::gemv_tile_scale_box_groups()), rows, CU_TENSOR_MAP_SWIZZLE_128B);
            };
            const int bk = q4::gemv_tile_box_k();
            auto encode_x = [&](CUtensorMap* mx) {
                encode_2d(mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.x, static_cast<uint64_t>(bk),
                          static_cast<uint64_t>(p.M) * (K / bk), static_cast<uint64_t>(bk) * 4,
                          static_cast<uint32_t>(bk), static_cast<uint32_t>(K / S / bk), CU_TENSOR_MAP_SWIZZLE_NONE);
            };
            if (p.maps != nullptr) {
                std::lock_guard<std::mutex> lk(p.maps->mu);
                if (p.maps->tile_rows != rows) {
                    encode_ws(&p.maps->tile_w, &p.maps->tile_s);
                    p.maps->tile_rows = rows;
                }
                if (p.maps->x_ptr != p.x || p.maps->x_m != p.M || p.maps->x_split != S) {
                    encode_x(&p.maps->tile_x);
                    p.maps->x_ptr = p.x;
                    p.maps->x_m = p.M;
                    p.maps->x_split = S;
                }
                a.tmap_w = p.maps->tile_w;
                a.tmap_s = p.maps->tile_s;
                a.tmap_x = p.maps->tile_x;
            } else {
                encode_ws(&a.tmap_w, &a.tmap_s);
                encode_x(&a.tmap_x);
            }
            a.y = p.y;
            a.M = p.M; a.N = N; a.K = K;
            a.cluster_k = S;
            a.lora_t = lora_t; a.lora_b = p.rank > 0 ? p.lora_b : nullptr; a.rank = p.rank; a.lora_scale = lscale;
            a.status = c.status;
            check_launch(q4::launch_gemv_tile(a, stream), "gemv tile launch");
            return;
        }
    }
    if (p.M <= 8 && dv == 2) {
        const int S = q4::decode_split(p.M, p.K);
        const int R = q4::decode_rows();
        const int waves_cl = S > 0 ? q4::decode_max_clusters(p.M, p.K, S, R) : 0;
        if (S > 0 && waves_cl > 0 && aligned16(p.x) && aligned16(p.packed) && aligned16(p.scales)) {
            // one wave of clusters while blocks stay <= 128 columns (>= 8 each)
            int G = std::min(waves_cl, std::max(1, p.N / 8));
            G = std::max(G, (p.N + R - 1) / R);
            const int rows = ((p.N + G - 1) / G + 7) / 8 * 8;
            q4::DecodeArgs a{};
            encode_2d(&a.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.packed, static_cast<uint64_t>(p.K) / 8,
                      static_cast<uint64_t>(p.N), static_cast<uint64_t>(p.K) / 2, 32, static_cast<uint32_t>(rows),
                      CU_TENSOR_MAP_SWIZZLE_128B);
            const int bx = q4::decode_x_box();
            encode_2d(&a.tmap_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.x, static_cast<uint64_t>(bx),
                      static_cast<uint64_t>(p.M) * (p.K / bx), static_cast<uint64_t>(bx) * 4,
                      static_cast<uint32_t>(bx), static_cast<uint32_t>(p.K / S / bx), CU_TENSOR_MAP_SWIZZLE_NONE);
            a.scales = p.scales; a.y = p.y;
            a.M = p.M; a.N = p.N; a.K = p.K;
            a.cluster_k = S; a.col_blocks = G; a.box_rows = rows;
            a.lora_t = lora_t; a.lora_b = p.rank > 0 ? p.lora_b : nullptr; a.rank = p.rank; a.lora_scale = lscale;
            a.status = c.status;
            check_launch(q4::launch_decode(a, stream), "decode launch");
            return;
        }
    }
    GemvGeom geo;
    if (p.M <= 8 && choose_gemv(c, p.M, p.N, p.K, geo)) {
        q4::GemvArgs a{};
        const int GS = p.K / 32 / geo.S;
        encode_2d(&a.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.packed, static_cast<uint64_t>(p.K) / 8,
                  static_cast<uint64_t>(p.N), static_cast<uint64_t>(p.K) / 2, static_cast<uint32_t>(GS * 4),
                  static_cast<uint32_t>(q4::gemv_chunk_columns()), CU_TENSOR_MAP_SWIZZLE_NONE);
        a.x = p.x; a.scales = p.scales; a.y = p.y;
        a.M = p.M; a.N = p.N; a.K = p.K;
        a.cluster_k = geo.S; a.clusters = geo.clusters; a.cols_per_cluster = geo.cols;
        a.lora_t = lora_t; a.lora_b = p.rank > 0 ? p.lora_b : nullptr; a.rank = p.rank; a.lora_scale = lscale;
        a.status = c.status;
        check_launch(q4::launch_gemv(a, stream), "gemv launch");
        return;
    }

    const q4::Operand16 op = operand_type();
    const bool f16 = op == q4::Operand16::kF16;
    // Variant: the CTA-pair kernel where use_pair_kernel allows it; else the
    // single-CTA kernel with 256-row tiles when they fill every SM; else
    // 128-row tiles.
    int pairs = 0;
    const int variant = g_gemm_variant.load();
    const bool use_pair = use_pair_kernel(c, p, op, &pairs);
    const int ksplit = use_pair && p.npeers == 0 ? pair_ksplit(p, pairs) : 1;  // pushes need whole tiles
    const long long ld_y = p.ld_y ? p.ld_y : p.N;
    if (ld_y != p.N && !use_pair) throw CudaError("strided Y reached a kernel without a row pitch");
    if (ksplit > 1)  // the K halves reduce-add into Y: zero it first (before the cast, so PDL still overlaps)
        check(cudaMemset2DAsync(p.y, static_cast<size_t>(ld_y) * 4, 0, static_cast<size_t>(p.N) * 4,
                                static_cast<size_t>(p.M), stream),
              "cudaMemset2DAsync (split-K Y)");
    Scratch x16(static_cast<size_t>(p.M) * p.K * 2, stream);
    Scratch rexp(f16 ? static_cast<size_t>(p.M) * sizeof(int) : 0, stream);
    Scratch cexp(f16 && p.col_exp == nullptr ? static_cast<size_t>(p.N) * sizeof(int) : 0, stream);
    int* row_exp = static_cast<int*>(rexp.p);
    const int* col_exp = f16 ? (p.col_exp ? p.col_exp : static_cast<int*>(cexp.p)) : nullptr;
    // Launches that do not need the cast go first, so that the cast is the
    // GEMM's direct predecessor and the GEMM's prologue (weights, dequant)
    // overlaps it through programmatic dependent launch: the per-column
    // exponents of a stateless call, and the pair kernel's fp32 T = X A (its
    // epilogue adds (alpha/r) T B).
    if (f16 && p.col_exp == nullptr)
        check_launch(q4::launch_col_exp(p.scales, static_cast<int*>(cexp.p), p.N, p.K, stream), "col_exp");
    // With split K the halves reduce-add into Y, so the LoRA term can come
    // after them: T = X A then runs on the helper stream beside the cast and
    // the GEMM (on the SMs the GEMM's units leave free), and one kernel adds
    // (alpha/r) T B once both are done.  Measured at configs[3] (M = 512):
    // 46.4 us per call against 50.8 us with the projection before the cast
    // (forking after the cast instead: 48.4 us).
    const bool lora_after = p.rank > 0 && use_pair && ksplit > 1;
    std::unique_lock<std::mutex> aux_lock;
    std::unique_ptr<CallEvent> fork_ev, join_ev;
    if (lora_after) {
        aux_lock = std::unique_lock<std::mutex>(c.aux_mu);
        const cudaStream_t aux = aux_stream(c);
        fork_ev = std::make_unique<CallEvent>();
        join_ev = std::make_unique<CallEvent>();
        check(cudaEventRecord(fork_ev->e, stream), "cudaEventRecord (fork)");
        check(cudaStreamWaitEvent(aux, fork_ev->e, 0), "cudaStreamWaitEvent (fork)");
        check_launch(q4::launch_lora_xa(p.x, p.lora_a, lora_t, p.M, p.K, p.rank, aux, static_cast<float*>(t_part.p)),
                     "lora_xa");
        check(cudaEventRecord(join_ev->e, aux), "cudaEventRecord (join)");
    } else if (p.rank > 0 && use_pair) {
        check_launch(q4::launch_lora_xa(p.x, p.lora_a, lora_t, p.M, p.K, p.rank, stream,
                                        static_cast<float*>(t_part.p)),
                     "lora_xa");
    }
    check_launch(q4::launch_cast_x(p.x, x16.p, row_exp, p.M, p.K, op, stream), "cast_x");

    q4::GemmArgs g{};
    g.ksplit = ksplit;
    g.halves = use_pair ? 1 : (variant == 3 || (variant == 0 && q4::gemm_tiles(p.M, p.N, 2) >= c.sm_count) ? 2 : 1);
    g.sm_count = p.sm_budget > 0 && p.sm_budget < c.sm_count ? p.sm_budget : c.sm_count;
    encode_2d(&g.tmap_x16, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x16.p,
              static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.M), static_cast<uint64_t>(p.K) * 2, 64,
              static_cast<uint32_t>(128 * g.halves), CU_TENSOR_MAP_SWIZZLE_128B);
    // packed W: 64-k boxes for the single-CTA kernel, 128-k boxes (64 B per
    // column, 64-byte swizzled) for the pair kernel
    encode_2d(&g.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.packed, static_cast<uint64_t>(p.K) / 8,
              static_cast<uint64_t>(p.N), static_cast<uint64_t>(p.K) / 2, use_pair ? 16 : 8, 128,
              use_pair ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE);
    if (use_pair) {
        encode_2d(&g.tmap_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.scales, static_cast<uint64_t>(p.K) / 32,
                  static_cast<uint64_t>(p.N), static_cast<uint64_t>(p.K) / 8, 4, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
        encode_2d(&g.tmap_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.y, static_cast<uint64_t>(p.N),
                  static_cast<uint64_t>(p.M), static_cast<uint64_t>(ld_y) * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    g.scales = p.scales; g.col_exp = col_exp; g.row_exp = row_exp; g.y = p.y;
    g.M = p.M; g.N = p.N; g.K = p.K; g.op = op;
    g.lora_b = p.rank > 0 && !lora_after ? p.lora_b : nullptr; g.rank = lora_after ? 0 : p.rank;
    g.lora_scale = lscale;
    g.status = c.status;
    if (p.npeers > 0) {
        g.peers = *p.peers;
        g.npeers = p.npeers;
        g.peer_ld = ld_y;
    }
    const int lstages = use_pair ? 0 : (p.rank + 15) / 16;
    Scratch t_op(lstages > 0 ? static_cast<size_t>(p.M) * lstages * 64 * 2 : 0, stream);
    if (p.rank > 0 && use_pair) {
        // T = X * A in fp32 (launched before the cast, above)
        g.tmap_t = g.tmap_x16;  // never read
        g.lora_t = lora_t;
        g.lora_stages = 0;
    } else if (p.rank > 0) {
        // T = X * A and its bf16 [hi | lo | hi | 0] operand scaled by the row exponents
        check_launch(q4::launch_lora_xa(p.x, p.lora_a, lora_t, p.M, p.K, p.rank, stream,
                                        static_cast<float*>(t_part.p), row_exp, static_cast<uint16_t*>(t_op.p)),
                     "lora_xa");
        encode_2d(&g.tmap_t, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, t_op.p, static_cast<uint64_t>(lstages) * 64,
                  static_cast<uint64_t>(p.M), static_cast<uint64_t>(lstages) * 128, 64,
                  static_cast<uint32_t>(128 * g.halves), CU_TENSOR_MAP_SWIZZLE_128B);
        g.lora_t = lora_t;
        g.lora_stages = use_pair ? 0 : lstages;
    } else {
        g.tmap_t = g.tmap_x16;  // never read
        g.lora_stages = 0;
    }
    if (use_pair)
        check_launch(q4::launch_gemm_pair(g, pairs, stream), "gemm (CTA pair) launch");
    else
        check_launch(q4::launch_gemm(g, stream), "gemm launch");
    if (lora_after) {
        check(cudaStreamWaitEvent(stream, join_ev->e, 0), "cudaStreamWaitEvent (join)");
        check_launch(q4::launch_lora_add(lora_t, p.lora_b, p.y, p.M, p.N, ld_y, p.rank, lscale, stream), "lora_add");
    }
}

// Reads and clears the status word (synchronises `stream` first).
// The status word rides on the same stream as the call's own copies, so one
// synchronisation covers both (no second round trip per call).  With
// `enqueued`, the call's copy-out kernel has already written it to the mapped
// host word.
// Waits until a host call's last kernel has set c.done_host (it does so after
// every one of its stores, Y and the status word, is visible to the host):
// about 2.5 us sooner than a stream synchronisation on this hardware.  Every
// 1024 polls the stream is queried; an error, an idle stream, or a second
// without the word ends the polling in a stream synchronisation, which
// reports the error or waits for the rest.
void wait_done(DeviceCtx& c) {
    volatile int* flag = c.done_host;
    const auto t0 = std::chrono::steady_clock::now();
    for (uint32_t i = 1;; ++i) {
        if (*flag) return;
#if defined(__x86_64__) || defined(__i386__)
        __builtin_ia32_pause();  // a spin-wait hint to the core; costs well under 0.1 us
#endif
        if ((i & 1023u) == 0) {
            if (cudaStreamQuery(c.stream) != cudaErrorNotReady) break;
            if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(1)) break;
        }
    }
    check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
}

// The status word of the work on `stream` (cleared on the device when set).
// enqueued: the work already copies it into c.status_host; done_flag: and
// then sets c.done_host, which the host waits on instead of the stream.
int take_status(DeviceCtx& c, cudaStream_t stream, bool enqueued = false, bool done_flag = false) {
    if (!enqueued)
        check(cudaMemcpyAsync(c.status_host, c.status, sizeof(int), cudaMemcpyDeviceToHost, stream), "read status");
    if (done_flag && stream == c.stream)
        wait_done(c);
    else
        check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    const int st = *static_cast<volatile int*>(c.status_host);
    if (st) {
        check(cudaMemsetAsync(c.status, 0, sizeof(int), stream), "clear status");
        check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    }
    return st;
}

// The address on the current device of a pinned, mapped host buffer (any
// page-locked allocation under unified addressing), or nullptr for pageable
// memory.
void* mapped_device_pointer(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();  // a plain pageable pointer on older drivers
        return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

// Device staging for a host-pointer call, kept per device and grown on
// demand (caller holds c.host_mu).
void* host_staging(DeviceCtx& c, size_t bytes) {
    if (bytes > c.hbuf_bytes) {
        if (c.hbuf) {
            check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
            cudaFree(c.hbuf);
            c.hbuf = nullptr;
            c.hbuf_bytes = 0;
        }
        const size_t want = std::max(bytes, static_cast<size_t>(1) << 20);
        check(cudaMalloc(&c.hbuf, want), "cudaMalloc host-call staging");
        c.hbuf_bytes = want;
        ++c.hbuf_gen;
    }
    return c.hbuf;
}

template <typename F>
int guarded(F&& f) {
    try {
        return f();
    } catch (const CudaError& e) {
        return fail(SPACESLUG_RUNTIME_FAILURE, e.what());
    } catch (const std::bad_alloc&) {
        return fail(SPACESLUG_RUNTIME_FAILURE, "host allocation failed");
    } catch (const std::exception& e) {
        return fail(SPACESLUG_RUNTIME_FAILURE, e.what());
    } catch (...) {
        return fail(SPACESLUG_RUNTIME_FAILURE, "unknown failure");
    }
}

void h2d(void* dst, const void* src, size_t bytes, cudaStream_t s) {
    if (bytes) check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s), "cudaMemcpyAsync H2D");
}
void d2h(void* dst, const void* src, size_t bytes, cudaStream_t s) {
    if (bytes) check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync D2H");
}

}  // namespace

// Helpers shared with csrc/noalloc.cu (the no-allocation entry point).  They
// reuse the GEMV geometry and tensor-map encoding above without touching the
// per-device context, which allocates on first use.
namespace q4rt {
cudaError_t noalloc_take_status(int device, int* out);  // csrc/noalloc.cu
bool gemv_geometry(int sm_count, int M, int N, int K, int* S, int* clusters, int* cols) {
    DeviceCtx tmp;
    tmp.sm_count = sm_count;
    GemvGeom geo;
    if (!choose_gemv(tmp, M, N, K, geo)) return false;
    *S = geo.S;
    *clusters = geo.clusters;
    *cols = geo.cols;
    return true;
}

bool encode_gemv_weights(CUtensorMap* map, const uint32_t* packed, int N, int K, int S) {
    try {
        encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, packed, static_cast<uint64_t>(K) / 8,
                  static_cast<uint64_t>(N), static_cast<uint64_t>(K) / 2, static_cast<uint32_t>(K / 32 / S * 4),
                  static_cast<uint32_t>(q4::gemv_chunk_columns()), CU_TENSOR_MAP_SWIZZLE_NONE);
        return true;
    } catch (...) {
        return false;
    }
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int set_error(int code, const char* msg) { return fail(code, msg); }
}  // namespace q4rt

struct spaceslug_q4_weights {
    int device = 0;
    int K = 0, N = 0;  // N = number of kept columns
    uint32_t col_begin = 0, n_total = 0;
    uint32_t* packed = nullptr;
    float* scales = nullptr;
    int* col_exp = nullptr;
    float* lora_a = nullptr;
    float* lora_b = nullptr;
    int rank = 0;
    float alpha = 0.0f;
    int sm_budget = 0;  // SMs a GEMM launch of this handle may occupy (0: all)
    DecodeMapCache decode_maps;  // tensor maps of its decode launches
    // Host-pointer calls with small pinned X and Y, captured once as a CUDA
    // graph (copy in, GEMV, copy out) and replayed: one graph launch instead
    // of three kernel launches per call.  Keyed by everything the captured
    // launches name; set_lora and destroy drop them.
    struct HostGraph {
        const float* x;
        float* y;
        const float* xmap;
        float* ymap;
        uint32_t m;
        int variant;
        uint64_t gen;
        cudaGraphExec_t exec;
    };

    std::vector<HostGraph> host_graphs;
    // training state (allocated on first use, reset by set_lora)
    float* lora_da = nullptr;
    float* lora_db = nullptr;
    float* adam = nullptr;  // first and second moments of A then of B: 2 * (K*r + r*N)
    int adam_step = 0;
};

// Caller holds the device's host_mu (or owns the handle exclusively).
void drop_host_graphs(spaceslug_q4_weights* w) {
    for (auto& g : w->host_graphs) cudaGraphExecDestroy(g.exec);
    w->host_graphs.clear();
}

// CQ4 (Cactus-Quants) matrix on one device: the indices repacked to the q4
// nibble order ([N][K/2] bytes), the norms expanded to one value per 32-k
// block ([N][K/32], the GEMM's scale grid), the codebook as 256 f16 pairs
// (codebook[b & 15], codebook[b >> 4]) for byte b of packed indices, and the
// activation-transform parameters.
struct spaceslug_cq4_weights {
    int device = 0;
    int K = 0, N = 0, gs = 0;
    bool orthogonal = false;
    float inv_sqrt = 1.0f;
    uint32_t* packed = nullptr;
    float* scales = nullptr;
    uint32_t* lut = nullptr;
    float* cbf = nullptr;  // codebook as fp32 [16] (decode rows)
    float* recip = nullptr;
    float* lsign = nullptr;
    float* rsign = nullptr;
    uint32_t* perm = nullptr;
    uint16_t* rotation = nullptr;
};

namespace {

// IEEE binary16 bits -> float (exact).
float half_bits_to_float(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            int e = -1;
            uint32_t m = man;
            do {
                ++e;
                m <<= 1;
            } while ((m & 0x400u) == 0);
            bits = sign | (static_cast<uint32_t>(127 - 15 - e) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// Codebook index of (n, k) in the stored layout (cactus_x86.cpp:25-53 and
// dequant_w.comp:45-97: LSB-first per (n, group), or 4-row interleaved panels).
uint32_t cq4_index(const spaceslug_cq4_matrix& m, bool orth, uint32_t n, uint32_t k) {
    const uint32_t gs = orth ? m.k : m.group_size, ng = orth ? 1u : m.num_groups;
    const uint32_t g = k / gs, kk = k % gs, pgb = gs / 2u;
    if (m.flags & SPACESLUG_CQ4_FLAG_INTERLEAVED_4ROW) {
        const uint8_t* panel = m.packed_indices + (static_cast<size_t>(n / 4u) * ng + g) * (4u * pgb);
        const uint8_t b = panel[(kk / 8u) * 16u + (n & 3u) * 4u + (kk & 3u)];
        return (kk & 4u) ? (b >> 4) : (b & 0xFu);
    }
    const uint8_t b = m.packed_indices[(static_cast<size_t>(n) * ng + g) * pgb + kk / 2u];
    return (b >> ((kk & 1u) * 4u)) & 0xFu;
}

float cq4_norm(const spaceslug_cq4_matrix& m, bool orth, uint32_t n, uint32_t g) {
    const bool il = (m.flags & SPACESLUG_CQ4_FLAG_INTERLEAVED_4ROW) != 0;
    size_t i;
    if (orth) i = il ? (n / 4u) * 4u + (n & 3u) : n;
    else i = il ? (static_cast<size_t>(n / 4u) * m.num_groups + g) * 4u + (n & 3u) : static_cast<size_t>(n) * m.num_groups + g;
    return half_bits_to_float(m.norms[i]);
}

void run_cq4(const spaceslug_cq4_weights& w, const void* a, void* c, int M, cudaStream_t stream) {
    DeviceCtx& ctx = ctx_for(current_device());
    const int K = w.K, N = w.N;
    q4::Cq4GemvArgs dv{a, w.packed, w.scales, w.cbf, w.recip, w.lsign, w.rsign, w.perm, w.inv_sqrt, 0, c, M, N, K};
    if (M <= 8 && static_cast<long long>(M) * K * 2 <= 192 * 1024 && !w.orthogonal) {
        // decode rows, Hadamard mode: one kernel (transform per CTA, then one warp per column), fp16 out
        dv.fused_gs = w.gs;
        check_launch(q4::launch_cq4_gemv(dv, stream), "cq4 gemv");
        return;
    }
    Scratch a1(static_cast<size_t>(M) * K * 2, stream);
    check_launch(q4::launch_cq4_transform(a, a1.p, w.recip, w.lsign, w.rsign, w.perm, w.rotation, M, K, w.gs,
                                          w.inv_sqrt, stream),
                 "cq4 transform");
    if (M <= 8 && static_cast<long long>(M) * K * 2 <= 192 * 1024) {
        dv.a = a1.p;  // orthogonal: the rotation ran as its own kernel
        check_launch(q4::launch_cq4_gemv(dv, stream), "cq4 gemv");
        return;
    }
    q4::GemmArgs g{};
    g.halves = q4::gemm_tiles(M, N, 2) >= ctx.sm_count ? 2 : 1;
    g.sm_count = ctx.sm_count;
    encode_2d(&g.tmap_x16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a1.p, static_cast<uint64_t>(K), static_cast<uint64_t>(M),
              static_cast<uint64_t>(K) * 2, 64, static_cast<uint32_t>(128 * g.halves), CU_TENSOR_MAP_SWIZZLE_128B);
    encode_2d(&g.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, w.packed, static_cast<uint64_t>(K) / 8,
              static_cast<uint64_t>(N), static_cast<uint64_t>(K) / 2, 8, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
    g.tmap_t = g.tmap_x16;  // never read
    g.scales = w.scales;
    g.y = nullptr;
    g.M = M; g.N = N; g.K = K;
    g.op = q4::Operand16::kF16;
    g.lut = w.lut;
    g.y16 = c;  // fp16 straight from the epilogue
    g.status = ctx.status;
    check_launch(q4::launch_gemm(g, stream), "cq4 gemm launch");
}

}  // namespace

extern "C" {

int spaceslug_vector_add(const float* left, const float* right, float* output, size_t count) {
    if (!left || !right || !output) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    for (size_t i = 0; i < count; ++i) output[i] = left[i] + right[i];
    return SPACESLUG_OK;
}

int spaceslug_q4_pack(const int8_t* w_kn, uint32_t k, uint32_t n, uint32_t* packed_out) {
    if (!w_kn || !packed_out) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (k == 0 || n == 0 || k % 32u) return fail(SPACESLUG_INVALID_ARGUMENT, "k must be a positive multiple of 32, n > 0");
    return guarded([&] {
        // Column-major output: for each column, K/8 words of 8 nibbles each;
        // the K/8 output chunks are split over host threads.
        q4up::host_pack(w_kn, k, n, packed_out);
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_pack_device(const int8_t* w_kn, uint32_t k, uint32_t n, uint32_t* packed_out, void* stream) {
    if (!w_kn || !packed_out) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (k == 0 || n == 0 || k % 32u) return fail(SPACESLUG_INVALID_ARGUMENT, "k must be a positive multiple of 32, n > 0");
    return guarded([&] {
        ctx_for(current_device());
        check_launch(q4::launch_pack(w_kn, packed_out, static_cast<int>(k), static_cast<int>(n),
                                     static_cast<cudaStream_t>(stream)),
                     "pack launch");
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_dequant_device(const uint32_t* packed, const float* scales, uint32_t k, uint32_t n, float* w_kn_out,
                                void* stream) {
    if (!packed || !scales || !w_kn_out) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (k == 0 || n == 0 || k % 32u) return fail(SPACESLUG_INVALID_ARGUMENT, "k must be a positive multiple of 32, n > 0");
    if (!aligned16(packed)) return fail(SPACESLUG_INVALID_ARGUMENT, "packed must be 16-byte aligned");
    return guarded([&] {
        ctx_for(current_device());
        check_launch(q4::launch_dequant(packed, scales, w_kn_out, static_cast<int>(k), static_cast<int>(n),
                                        static_cast<cudaStream_t>(stream)),
                     "dequant launch");
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_dequant(const uint32_t* packed, const float* scales, uint32_t k, uint32_t n, float* w_kn_out) {
    if (!packed || !scales || !w_kn_out) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (k == 0 || n == 0 || k % 32u) return fail(SPACESLUG_INVALID_ARGUMENT, "k must be a positive multiple of 32, n > 0");
    return guarded([&] {
        DeviceCtx& c = ctx_for(current_device());
        std::lock_guard<std::mutex> lk(c.host_mu);
        const size_t pw = static_cast<size_t>(k) * n / 2, sb = static_cast<size_t>(n) * (k / 32) * 4,
                     wb = static_cast<size_t>(k) * n * 4;
        Scratch dp(pw, c.stream), ds(sb, c.stream), dw(wb, c.stream);
        h2d(dp.p, packed, pw, c.stream);
        h2d(ds.p, scales, sb, c.stream);
        check_launch(q4::launch_dequant(static_cast<uint32_t*>(dp.p), static_cast<float*>(ds.p),
                                        static_cast<float*>(dw.p), static_cast<int>(k), static_cast<int>(n), c.stream),
                     "dequant launch");
        d2h(w_kn_out, dw.p, wb, c.stream);
        check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        return SPACESLUG_OK;
    });
}

int spaceslug_q4gemm_device(const float* x, const uint32_t* packed, const float* scales, const float* lora_a,
                            const float* lora_b, uint32_t rank, float alpha, float* y, uint32_t m, uint32_t n,
                            uint32_t k, void* stream) {
    if (const char* err = shape_error(x, packed, scales, y, m, n, k, rank, lora_a, lora_b, alpha))
        return fail(SPACESLUG_INVALID_ARGUMENT, err);
    if (!aligned16(x) || !aligned16(packed) || !aligned16(y))
        return fail(SPACESLUG_INVALID_ARGUMENT, "x, packed and y must be 16-byte aligned");
    return guarded([&] {
        Problem p{x, packed, scales, nullptr, lora_a, lora_b, static_cast<int>(rank), alpha, y,
                  static_cast<int>(m), static_cast<int>(n), static_cast<int>(k)};
        run_problem(p, static_cast<cudaStream_t>(stream));
        return SPACESLUG_OK;
    });
}

int spaceslug_q4gemm_lora(const float* x, const uint32_t* packed, const float* scales, const float* lora_a,
                          const float* lora_b, uint32_t rank, float alpha, float* y, uint32_t m, uint32_t n,
                          uint32_t k) {
    if (const char* err = shape_error(x, packed, scales, y, m, n, k, rank, lora_a, lora_b, alpha))
        return fail(SPACESLUG_INVALID_ARGUMENT, err);
    if (rank == 0) return fail(SPACESLUG_INVALID_ARGUMENT, "LoRA rank must be >= 1");
    return guarded([&] {
        DeviceCtx& c = ctx_for(current_device());
        std::lock_guard<std::mutex> lk(c.host_mu);
        const size_t xb = static_cast<size_t>(m) * k * 4, pb = static_cast<size_t>(k) * n / 2,
                     sb = static_cast<size_t>(n) * (k / 32) * 4, yb = static_cast<size_t>(m) * n * 4,
                     ab = static_cast<size_t>(k) * rank * 4, bb = static_cast<size_t>(rank) * n * 4;
        Scratch dx(xb, c.stream), dp(pb, c.stream), ds(sb, c.stream), dy(yb, c.stream), da(ab, c.stream),
            db(bb, c.stream);
        h2d(dx.p, x, xb, c.stream);
        h2d(dp.p, packed, pb, c.stream);
        h2d(ds.p, scales, sb, c.stream);
        h2d(da.p, lora_a, ab, c.stream);
        h2d(db.p, lora_b, bb, c.stream);
        Problem p{static_cast<float*>(dx.p), static_cast<uint32_t*>(dp.p), static_cast<float*>(ds.p), nullptr,
                  static_cast<float*>(da.p), static_cast<float*>(db.p), static_cast<int>(rank), alpha,
                  static_cast<float*>(dy.p), static_cast<int>(m), static_cast<int>(n), static_cast<int>(k)};
        run_problem(p, c.stream);
        d2h(y, dy.p, yb, c.stream);
        if (take_status(c, c.stream)) return fail(SPACESLUG_TIMEOUT, "a kernel wait timed out");
        return SPACESLUG_OK;
    });
}

int spaceslug_q4gemm(const float* x, const uint32_t* packed, const float* scales, float* y, uint32_t m, uint32_t n,
                     uint32_t k) {
    if (const char* err = shape_error(x, packed, scales, y, m, n, k, 0, nullptr, nullptr, 0.0f))
        return fail(SPACESLUG_INVALID_ARGUMENT, err);
    return guarded([&] {
        DeviceCtx& c = ctx_for(current_device());
        std::lock_guard<std::mutex> lk(c.host_mu);
        const size_t xb = static_cast<size_t>(m) * k * 4, pb = static_cast<size_t>(k) * n / 2,
                     sb = static_cast<size_t>(n) * (k / 32) * 4, yb = static_cast<size_t>(m) * n * 4;
        Scratch dx(xb, c.stream), dp(pb, c.stream), ds(sb, c.stream), dy(yb, c.stream);
        h2d(dx.p, x, xb, c.stream);
        h2d(dp.p, packed, pb, c.stream);
        h2d(ds.p, scales, sb, c.stream);
        Problem p{static_cast<float*>(dx.p), static_cast<uint32_t*>(dp.p), static_cast<float*>(ds.p), nullptr,
                  nullptr, nullptr, 0, 0.0f, static_cast<float*>(dy.p), static_cast<int>(m), static_cast<int>(n),
                  static_cast<int>(k)};
        run_problem(p, c.stream);
        d2h(y, dy.p, yb, c.stream);
        if (take_status(c, c.stream)) return fail(SPACESLUG_TIMEOUT, "a kernel wait timed out");
        return SPACESLUG_OK;
    });
}

int spaceslug_lora_delta(const float* x, const float* a, const float* b, float* y, uint32_t m, uint32_t rank) {
    // Same checks as vulkan-runtime/src/api/lora_delta_api.cpp:44.
    if (x == nullptr || a == nullptr || b == nullptr || y == nullptr || m == 0 || m > 128 || rank == 0 || rank > 8)
        return fail(SPACESLUG_INVALID_ARGUMENT, "invalid arguments (need 1<=m<=128, 1<=rank<=8, non-null)");
    return guarded([&] {
        DeviceCtx& c = ctx_for(current_device());
        std::lock_guard<std::mutex> lk(c.host_mu);
        const size_t xb = static_cast<size_t>(m) * 64 * 4, ab = 64u * rank * 4, bb = rank * 64u * 4;
        Scratch dx(xb, c.stream), da(ab, c.stream), db(bb, c.stream), dy(xb, c.stream);
        h2d(dx.p, x, xb, c.stream);
        h2d(da.p, a, ab, c.stream);
        h2d(db.p, b, bb, c.stream);
        check_launch(q4::launch_lora_delta64(static_cast<float*>(dx.p), static_cast<float*>(da.p),
                                             static_cast<float*>(db.p), static_cast<float*>(dy.p),
                                             static_cast<int>(m), static_cast<int>(rank), c.stream),
                     "lora_delta launch");
        d2h(y, dy.p, xb, c.stream);
        check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_create(const uint32_t* packed, const float* scales, uint32_t k, uint32_t n,
                                uint32_t col_begin, uint32_t col_end, int device, spaceslug_q4_weights** out) {
    if (!packed || !scales || !out) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (k == 0 || n == 0 || k % 32u) return fail(SPACESLUG_INVALID_ARGUMENT, "k must be a positive multiple of 32, n > 0");
    if (col_begin >= col_end || col_end > n) return fail(SPACESLUG_INVALID_ARGUMENT, "bad column range");
    *out = nullptr;
    return guarded([&] {
        check(cudaSetDevice(device), "cudaSetDevice");
        DeviceCtx& c = ctx_for(device);
        auto* w = new spaceslug_q4_weights();
        w->device = device;
        w->K = static_cast<int>(k);
        w->N = static_cast<int>(col_end - col_begin);
        w->col_begin = col_begin;
        w->n_total = n;
        const size_t G = k / 32u;
        const size_t pb = static_cast<size_t>(w->N) * k / 2, sb = static_cast<size_t>(w->N) * G * 4;
        try {
            check(cudaMalloc(&w->packed, pb), "cudaMalloc packed");
            check(cudaMalloc(&w->scales, sb), "cudaMalloc scales");
            check(cudaMalloc(&w->col_exp, static_cast<size_t>(w->N) * sizeof(int)), "cudaMalloc col_exp");
            std::lock_guard<std::mutex> lk(c.host_mu);
            q4up::staged_h2d(device, w->packed, packed + static_cast<size_t>(col_begin) * (k / 8u), pb, c.stream);
            q4up::staged_h2d(device, w->scales, scales + static_cast<size_t>(col_begin) * G, sb, c.stream);
            check_launch(q4::launch_col_exp(w->scales, w->col_exp, w->N, w->K, c.stream), "col_exp");
            check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        } catch (...) {
            spaceslug_q4_weights_destroy(w);
            throw;
        }
        *out = w;
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_create_logical(const int8_t* w_kn, const float* scales, uint32_t k, uint32_t n,
                                        uint32_t col_begin, uint32_t col_end, int device, spaceslug_q4_weights** out) {
    if (!w_kn || !scales || !out) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (k == 0 || n == 0 || k % 32u) return fail(SPACESLUG_INVALID_ARGUMENT, "k must be a positive multiple of 32, n > 0");
    if (col_begin >= col_end || col_end > n) return fail(SPACESLUG_INVALID_ARGUMENT, "bad column range");
    *out = nullptr;
    return guarded([&] {
        check(cudaSetDevice(device), "cudaSetDevice");
        DeviceCtx& c = ctx_for(device);
        auto* w = new spaceslug_q4_weights();
        w->device = device;
        w->K = static_cast<int>(k);
        w->N = static_cast<int>(col_end - col_begin);
        w->col_begin = col_begin;
        w->n_total = n;
        const size_t G = k / 32u;
        const size_t pb = static_cast<size_t>(w->N) * k / 2, sb = static_cast<size_t>(w->N) * G * 4;
        try {
            check(cudaMalloc(&w->packed, pb), "cudaMalloc packed");
            check(cudaMalloc(&w->scales, sb), "cudaMalloc scales");
            check(cudaMalloc(&w->col_exp, static_cast<size_t>(w->N) * sizeof(int)), "cudaMalloc col_exp");
            std::lock_guard<std::mutex> lk(c.host_mu);
            q4up::staged_pack_logical(device, w->packed, w_kn, k, n, col_begin, static_cast<uint32_t>(w->N), c.stream);
            q4up::staged_h2d(device, w->scales, scales + static_cast<size_t>(col_begin) * G, sb, c.stream);
            check_launch(q4::launch_col_exp(w->scales, w->col_exp, w->N, w->K, c.stream), "col_exp");
            check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        } catch (...) {
            spaceslug_q4_weights_destroy(w);
            throw;
        }
        *out = w;
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_export(const spaceslug_q4_weights* w, uint32_t* packed_out, float* scales_out) {
    if (!w || (!packed_out && !scales_out)) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    return guarded([&] {
        check(cudaSetDevice(w->device), "cudaSetDevice");
        DeviceCtx& c = ctx_for(w->device);
        std::lock_guard<std::mutex> lk(c.host_mu);
        if (packed_out) d2h(packed_out, w->packed, static_cast<size_t>(w->N) * w->K / 2, c.stream);
        if (scales_out) d2h(scales_out, w->scales, static_cast<size_t>(w->N) * (w->K / 32) * 4, c.stream);
        check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_set_lora(spaceslug_q4_weights* w, const float* lora_a, const float* lora_b, uint32_t rank,
                                  float alpha) {
    if (!w) return fail(SPACESLUG_INVALID_ARGUMENT, "null handle");
    if (rank > 64) return fail(SPACESLUG_INVALID_ARGUMENT, "LoRA rank must be <= 64");
    if (rank > 0 && (!lora_a || !lora_b || !std::isfinite(alpha)))
        return fail(SPACESLUG_INVALID_ARGUMENT, "LoRA needs A, B and a finite alpha");
    return guarded([&] {
        check(cudaSetDevice(w->device), "cudaSetDevice");
        {
            // graphs of host calls name the old adapter's buffers and scale
            DeviceCtx& c = ctx_for(w->device);
            std::lock_guard<std::mutex> lk(c.host_mu);
            drop_host_graphs(w);
        }
        cudaFree(w->lora_a);
        cudaFree(w->lora_b);
        cudaFree(w->lora_da);
        cudaFree(w->lora_db);
        cudaFree(w->adam);
        w->lora_a = w->lora_b = w->lora_da = w->lora_db = w->adam = nullptr;
        w->adam_step = 0;
        w->rank = 0;
        if (rank == 0) return SPACESLUG_OK;
        // lora_b is the full [rank x n_total] matrix; keep the handle's columns.
        check(cudaMalloc(&w->lora_a, static_cast<size_t>(w->K) * rank * 4), "cudaMalloc lora_a");
        check(cudaMalloc(&w->lora_b, static_cast<size_t>(rank) * w->N * 4), "cudaMalloc lora_b");
        check(cudaMemcpy(w->lora_a, lora_a, static_cast<size_t>(w->K) * rank * 4, cudaMemcpyHostToDevice), "H2D A");
        check(cudaMemcpy2D(w->lora_b, static_cast<size_t>(w->N) * 4, lora_b + w->col_begin,
                           static_cast<size_t>(w->n_total) * 4, static_cast<size_t>(w->N) * 4, rank,
                           cudaMemcpyHostToDevice),
              "H2D B");
        w->rank = static_cast<int>(rank);
        w->alpha = alpha;
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_run(spaceslug_q4_weights* w, const float* x, float* y, uint32_t m, void* stream) {
    if (!w || !x || !y) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (m == 0 || m > (1u << 30)) return fail(SPACESLUG_INVALID_ARGUMENT, "bad m");
    if (!aligned16(x) || !aligned16(y)) return fail(SPACESLUG_INVALID_ARGUMENT, "x and y must be 16-byte aligned");
    return guarded([&] {
        if (current_device() != w->device) check(cudaSetDevice(w->device), "cudaSetDevice");
        Problem p{x, w->packed, w->scales, w->col_exp, w->lora_a, w->lora_b, w->rank, w->alpha, y,
                  static_cast<int>(m), w->N, w->K};
        p.sm_budget = w->sm_budget;
        p.maps = &w->decode_maps;
        run_problem(p, static_cast<cudaStream_t>(stream));
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_run_strided(spaceslug_q4_weights* w, const float* x, float* y, uint32_t m, uint64_t ld_y,
                                     void* stream) {
    if (!w || !x || !y) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (m == 0 || m > (1u << 30)) return fail(SPACESLUG_INVALID_ARGUMENT, "bad m");
    if (ld_y < static_cast<uint64_t>(w->N) || ld_y > (uint64_t(1) << 40))
        return fail(SPACESLUG_INVALID_ARGUMENT, "ld_y must be >= the handle's column count");
    if (!aligned16(x) || (reinterpret_cast<uintptr_t>(y) & 3u))
        return fail(SPACESLUG_INVALID_ARGUMENT, "x must be 16-byte and y 4-byte aligned");
    return guarded([&] {
        if (current_device() != w->device) check(cudaSetDevice(w->device), "cudaSetDevice");
        Problem p{x, w->packed, w->scales, w->col_exp, w->lora_a, w->lora_b, w->rank, w->alpha, y,
                  static_cast<int>(m), w->N, w->K, static_cast<long long>(ld_y), w->sm_budget};
        if (ld_y == static_cast<uint64_t>(w->N) && !aligned16(y)) {
            // the kernels want a 16-byte aligned Y: product in scratch, then one copy
            // (a pitched, unaligned Y takes the same route inside run_problem)
            Scratch ys(static_cast<size_t>(m) * w->N * 4, static_cast<cudaStream_t>(stream));
            Problem q = p;
            q.y = static_cast<float*>(ys.p);
            q.ld_y = 0;
            run_problem(q, static_cast<cudaStream_t>(stream));
            check(cudaMemcpyAsync(y, ys.p, static_cast<size_t>(m) * w->N * 4, cudaMemcpyDeviceToDevice,
                                  static_cast<cudaStream_t>(stream)),
                  "cudaMemcpyAsync (unaligned Y)");
            return SPACESLUG_OK;
        }
        run_problem(p, static_cast<cudaStream_t>(stream));
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_set_sm_budget(spaceslug_q4_weights* w, uint32_t sms) {
    if (!w) return fail(SPACESLUG_INVALID_ARGUMENT, "null handle");
    if (sms == 1 || sms > 4096) return fail(SPACESLUG_INVALID_ARGUMENT, "sms must be 0 (all) or 2..4096");
    w->sm_budget = static_cast<int>(sms);
    return SPACESLUG_OK;
}

int spaceslug_push_rows(const float* src, float* const* peer_dst, uint32_t npeers, uint32_t rows, uint32_t width,
                        uint64_t ld, uint32_t ctas, void* stream) {
    if (!src || (npeers && !peer_dst)) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (npeers > static_cast<uint32_t>(q4::kMaxPeers)) return fail(SPACESLUG_INVALID_ARGUMENT, "at most 7 peers");
    if (width == 0 || ld < width || ld > (uint64_t(1) << 40) || rows > (1u << 30) || width > (1u << 30))
        return fail(SPACESLUG_INVALID_ARGUMENT, "bad width / ld / rows");
    if (ctas == 0 || ctas > 65535) return fail(SPACESLUG_INVALID_ARGUMENT, "ctas must be 1..65535");
    q4::PeerPtrs pp{};
    for (uint32_t q = 0; q < npeers; ++q) {
        if (!peer_dst[q]) return fail(SPACESLUG_INVALID_ARGUMENT, "null peer pointer");
        pp.p[q] = peer_dst[q];
    }
    if (npeers == 0 || rows == 0) return SPACESLUG_OK;
    return guarded([&] {
        check_launch(q4::launch_push_rows(src, pp, static_cast<int>(npeers), static_cast<int>(rows),
                                          static_cast<int>(width), static_cast<long long>(ld), static_cast<int>(ctas),
                                          static_cast<cudaStream_t>(stream)),
                     "push_rows");
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_run_push(spaceslug_q4_weights* w, const float* x, float* y, uint32_t m, uint64_t ld_y,
                                  float* const* peer_y, uint32_t npeers, void* stream) {
    if (!w || !x || !y || (npeers && !peer_y)) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (m == 0 || m > (1u << 30)) return fail(SPACESLUG_INVALID_ARGUMENT, "bad m");
    if (npeers > static_cast<uint32_t>(q4::kMaxPeers)) return fail(SPACESLUG_INVALID_ARGUMENT, "at most 7 peers");
    if (ld_y < static_cast<uint64_t>(w->N) || ld_y > (uint64_t(1) << 40))
        return fail(SPACESLUG_INVALID_ARGUMENT, "ld_y must be >= the handle's column count");
    if (!aligned16(x) || (reinterpret_cast<uintptr_t>(y) & 3u))
        return fail(SPACESLUG_INVALID_ARGUMENT, "x must be 16-byte and y 4-byte aligned");
    q4::PeerPtrs pp{};
    for (uint32_t q = 0; q < npeers; ++q) {
        if (!peer_y[q] || (reinterpret_cast<uintptr_t>(peer_y[q]) & 3u))
            return fail(SPACESLUG_INVALID_ARGUMENT, "null or misaligned peer pointer");
        pp.p[q] = peer_y[q];
    }
    return guarded([&] {
        if (current_device() != w->device) check(cudaSetDevice(w->device), "cudaSetDevice");
        Problem p{x, w->packed, w->scales, w->col_exp, w->lora_a, w->lora_b, w->rank, w->alpha, y,
                  static_cast<int>(m), w->N, w->K, static_cast<long long>(ld_y), w->sm_budget};
        p.peers = &pp;
        p.npeers = static_cast<int>(npeers);
        run_problem(p, static_cast<cudaStream_t>(stream));
        return SPACESLUG_OK;
    });
}

int spaceslug_ipc_export(const void* ptr, void* handle64, uint64_t* offset) {
    if (!ptr || !handle64 || !offset) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    return guarded([&] {
        cudaPointerAttributes a{};
        check(cudaPointerGetAttributes(&a, ptr), "cudaPointerGetAttributes");
        if (a.type != cudaMemoryTypeDevice) throw CudaError("not device memory");
        using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
        static RangeFn range = [] {
            void* fn = nullptr;
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
                q != cudaDriverEntryPointSuccess)
                fn = nullptr;
            return reinterpret_cast<RangeFn>(fn);
        }();
        if (!range) throw CudaError("cuMemGetAddressRange is unavailable");
        const int prev = current_device();
        check(cudaSetDevice(a.device), "cudaSetDevice");
        CUdeviceptr base = 0;
        size_t size = 0;
        const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
        if (r != CUDA_SUCCESS) {
            cudaSetDevice(prev);
            throw CudaError("cuMemGetAddressRange failed (" + std::to_string(static_cast<int>(r)) + ")");
        }
        cudaIpcMemHandle_t h;
        const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
        cudaSetDevice(prev);
        check(e, "cudaIpcGetMemHandle");
        static_assert(sizeof(h) == 64, "IPC handle size");
        std::memcpy(handle64, &h, sizeof(h));
        *offset = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
        return SPACESLUG_OK;
    });
}

int spaceslug_ipc_open(const void* handle64, uint64_t offset, int device, void** ptr, void** base) {
    if (!handle64 || !ptr || !base) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    *ptr = *base = nullptr;
    return guarded([&] {
        check(cudaSetDevice(device), "cudaSetDevice");
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handle64, sizeof(h));
        void* b = nullptr;
        check(cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
        *base = b;
        *ptr = static_cast<char*>(b) + offset;
        return SPACESLUG_OK;
    });
}

int spaceslug_ipc_close(void* base) {
    if (!base) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    return guarded([&] {
        check(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
        return SPACESLUG_OK;
    });
}

int spaceslug_copy_2d(void* dst, uint64_t dpitch, const void* src, uint64_t spitch, uint64_t width_bytes,
                      uint64_t rows, void* stream) {
    if (!dst || !src) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (width_bytes > dpitch || width_bytes > spitch) return fail(SPACESLUG_INVALID_ARGUMENT, "width exceeds a pitch");
    if (width_bytes == 0 || rows == 0) return SPACESLUG_OK;
    return guarded([&] {
        check(cudaMemcpy2DAsync(dst, dpitch, src, spitch, width_bytes, rows, cudaMemcpyDefault,
                                static_cast<cudaStream_t>(stream)),
              "cudaMemcpy2DAsync");
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_run_host(spaceslug_q4_weights* w, const float* x, float* y, uint32_t m) {
    if (!w || !x || !y) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (m == 0 || m > (1u << 30)) return fail(SPACESLUG_INVALID_ARGUMENT, "bad m");
    return guarded([&] {
        check(cudaSetDevice(w->device), "cudaSetDevice");
        DeviceCtx& c = ctx_for(w->device);
        std::lock_guard<std::mutex> lk(c.host_mu);
        const size_t xb = static_cast<size_t>(m) * w->K * 4, yb = static_cast<size_t>(m) * w->N * 4;
        const size_t yoff = (xb + 255) / 256 * 256;
        char* stage = static_cast<char*>(host_staging(c, yoff + yb));
        float* dx = reinterpret_cast<float*>(stage);
        float* dy = reinterpret_cast<float*>(stage + yoff);
        // Small pinned (mapped) host buffers move by copy kernels over the bus,
        // the status word with Y: a copy-engine transfer of a few kilobytes
        // costs ~8 us.  Pageable buffers, and pinned ones above
        // kZeroCopyMaxBytes (prefill-sized X and Y, where the copy engine's
        // bandwidth matters more than its latency), take copy-engine transfers.
        constexpr size_t kZeroCopyMaxBytes = size_t(1) << 20;
        const float* xmap = xb <= kZeroCopyMaxBytes ? static_cast<const float*>(mapped_device_pointer(x)) : nullptr;
        float* ymap = yb <= kZeroCopyMaxBytes ? static_cast<float*>(mapped_device_pointer(y)) : nullptr;
        auto issue = [&] {
            if (xmap)
                check_launch(q4::launch_copy_words(xmap, dx, static_cast<long long>(m) * w->K, nullptr, nullptr,
                                                   c.stream),
                             "copy X in");
            else
                h2d(dx, x, xb, c.stream);
            Problem p{dx, w->packed, w->scales, w->col_exp, w->lora_a, w->lora_b, w->rank, w->alpha, dy,
                      static_cast<int>(m), w->N, w->K};
            p.sm_budget = w->sm_budget;
            p.maps = &w->decode_maps;
            run_problem(p, c.stream);
            if (ymap)
                check_launch(q4::launch_copy_words(dy, ymap, static_cast<long long>(m) * w->N, c.status,
                                                   c.status_host_dev, c.stream, c.done_host_dev, c.done_count),
                             "copy Y out");
            else
                d2h(y, dy, yb, c.stream);
        };
        const int variant = decode_variant_init().load();
        if (ymap) *static_cast<volatile int*>(c.done_host) = 0;  // the copy-out kernel sets it again
        if (xmap && ymap && m <= 8) {
            // decode-sized call with pinned buffers: replay (or capture) its graph
            cudaGraphExec_t exec = nullptr;
            for (auto& g : w->host_graphs)
                if (g.x == x && g.y == y && g.xmap == xmap && g.ymap == ymap && g.m == m && g.variant == variant &&
                    g.gen == c.hbuf_gen) {
                    exec = g.exec;
                    break;
                }
            if (exec == nullptr) {
                // Capture once; anything the capture does not take (it should
                // take all of it) falls back to direct launches for this call.
                cudaGraph_t graph = nullptr;
                bool captured = false;
                if (cudaStreamBeginCapture(c.stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
                    try {
                        issue();
                        captured = true;
                    } catch (...) {
                    }
                    if (cudaStreamEndCapture(c.stream, &graph) != cudaSuccess) captured = false;
                    if (captured && cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) {
                        captured = false;
                        exec = nullptr;
                    }
                    if (graph) cudaGraphDestroy(graph);
                }
                cudaGetLastError();  // a failed capture leaves no sticky error behind
                if (captured) {
                    if (w->host_graphs.size() >= 8) {  // keep the most recent few buffer pairs
                        cudaGraphExecDestroy(w->host_graphs.front().exec);
                        w->host_graphs.erase(w->host_graphs.begin());
                    }
                    w->host_graphs.push_back({x, y, xmap, ymap, m, variant, c.hbuf_gen, exec});
                }
            }
            if (exec != nullptr)
                check(cudaGraphLaunch(exec, c.stream), "cudaGraphLaunch");
            else
                issue();
        } else {
            issue();
        }
        if (take_status(c, c.stream, ymap != nullptr, ymap != nullptr))
            return fail(SPACESLUG_TIMEOUT, "a kernel wait timed out");
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_destroy(spaceslug_q4_weights* w) {
    if (!w) return fail(SPACESLUG_INVALID_ARGUMENT, "null handle");
    cudaSetDevice(w->device);
    {
        DeviceCtx& c = g_ctx[w->device];
        std::lock_guard<std::mutex> lk(c.host_mu);
        drop_host_graphs(w);
    }
    cudaFree(w->packed);
    cudaFree(w->scales);
    cudaFree(w->col_exp);
    cudaFree(w->lora_a);
    cudaFree(w->lora_b);
    cudaFree(w->lora_da);
    cudaFree(w->lora_db);
    cudaFree(w->adam);
    delete w;
    return SPACESLUG_OK;
}

int spaceslug_lora_gradients(const float* x, const float* dy, const float* a, const float* b, float* da, float* db,
                             uint32_t m, uint32_t rank) {
    // Same checks as vulkan-runtime/src/api/lora_gradients_api.cpp:23.
    if (!x || !dy || !a || !b || !da || !db || m == 0 || m > 128 || rank == 0 || rank > 8)
        return fail(SPACESLUG_INVALID_ARGUMENT, "invalid arguments (need 1<=m<=128, 1<=rank<=8, non-null)");
    return guarded([&] {
        DeviceCtx& c = ctx_for(current_device());
        std::lock_guard<std::mutex> lk(c.host_mu);
        const int M = static_cast<int>(m), r = static_cast<int>(rank);
        const size_t xb = static_cast<size_t>(M) * 64 * 4, pb = 64u * rank * 4;
        Scratch dx(xb, c.stream), ddy(xb, c.stream), dA(pb, c.stream), dB(pb, c.stream), gA(pb, c.stream),
            gB(pb, c.stream), sc(q4::lora_backward_scratch_floats(M, 64, 64, r) * 4, c.stream);
        h2d(dx.p, x, xb, c.stream);
        h2d(ddy.p, dy, xb, c.stream);
        h2d(dA.p, a, pb, c.stream);
        h2d(dB.p, b, pb, c.stream);
        q4::LoraBackwardArgs g{static_cast<float*>(dx.p), static_cast<float*>(ddy.p), static_cast<float*>(dA.p),
                               static_cast<float*>(dB.p), static_cast<float*>(gA.p), static_cast<float*>(gB.p),
                               static_cast<float*>(sc.p), M, 64, 64, r, 1.0f};
        check_launch(q4::launch_lora_backward(g, c.stream), "lora backward");
        d2h(da, gA.p, pb, c.stream);
        d2h(db, gB.p, pb, c.stream);
        check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        return SPACESLUG_OK;
    });
}

int spaceslug_lora_sgd(float* a, float* b, const float* da, const float* db, float learning_rate, uint32_t rank) {
    // Same checks as vulkan-runtime/src/api/lora_sgd_api.cpp:23.
    if (!a || !b || !da || !db || !(learning_rate > 0.0f) || rank == 0 || rank > 8)
        return fail(SPACESLUG_INVALID_ARGUMENT, "invalid arguments (need learning_rate > 0, 1<=rank<=8, non-null)");
    return guarded([&] {
        DeviceCtx& c = ctx_for(current_device());
        std::lock_guard<std::mutex> lk(c.host_mu);
        const size_t pb = 64u * rank * 4;
        Scratch dA(pb, c.stream), dB(pb, c.stream), gA(pb, c.stream), gB(pb, c.stream);
        h2d(dA.p, a, pb, c.stream);
        h2d(dB.p, b, pb, c.stream);
        h2d(gA.p, da, pb, c.stream);
        h2d(gB.p, db, pb, c.stream);
        check_launch(q4::launch_sgd(static_cast<float*>(dA.p), static_cast<float*>(gA.p), learning_rate, 64 * rank,
                                    c.stream),
                     "sgd A");
        check_launch(q4::launch_sgd(static_cast<float*>(dB.p), static_cast<float*>(gB.p), learning_rate, 64 * rank,
                                    c.stream),
                     "sgd B");
        d2h(a, dA.p, pb, c.stream);
        d2h(b, dB.p, pb, c.stream);
        check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        return SPACESLUG_OK;
    });
}

int spaceslug_lora_train_step(const float* x, const float* dy, float* a, float* b, float* y, float learning_rate,
                              uint32_t m, uint32_t rank) {
    // Same checks as vulkan-runtime/src/api/lora_train_api.cpp:10; the same
    // sequence (delta forward, gradients at the old A/B, SGD) on the device.
    if (!x || !dy || !a || !b || !y || !(learning_rate > 0.0f) || m == 0 || m > 128 || rank == 0 || rank > 8)
        return fail(SPACESLUG_INVALID_ARGUMENT, "invalid arguments (need learning_rate > 0, 1<=m<=128, 1<=rank<=8)");
    return guarded([&] {
        DeviceCtx& c = ctx_for(current_device());
        std::lock_guard<std::mutex> lk(c.host_mu);
        const int M = static_cast<int>(m), r = static_cast<int>(rank);
        const size_t xb = static_cast<size_t>(M) * 64 * 4, pb = 64u * rank * 4;
        Scratch dx(xb, c.stream), ddy(xb, c.stream), dyo(xb, c.stream), dA(pb, c.stream), dB(pb, c.stream),
            gA(pb, c.stream), gB(pb, c.stream), sc(q4::lora_backward_scratch_floats(M, 64, 64, r) * 4, c.stream);
        h2d(dx.p, x, xb, c.stream);
        h2d(ddy.p, dy, xb, c.stream);
        h2d(dA.p, a, pb, c.stream);
        h2d(dB.p, b, pb, c.stream);
        check_launch(q4::launch_lora_delta64(static_cast<float*>(dx.p), static_cast<float*>(dA.p),
                                             static_cast<float*>(dB.p), static_cast<float*>(dyo.p), M, r, c.stream),
                     "lora_delta launch");
        q4::LoraBackwardArgs g{static_cast<float*>(dx.p), static_cast<float*>(ddy.p), static_cast<float*>(dA.p),
                               static_cast<float*>(dB.p), static_cast<float*>(gA.p), static_cast<float*>(gB.p),
                               static_cast<float*>(sc.p), M, 64, 64, r, 1.0f};
        check_launch(q4::launch_lora_backward(g, c.stream), "lora backward");
        check_launch(q4::launch_sgd(static_cast<float*>(dA.p), static_cast<float*>(gA.p), learning_rate, 64 * r, c.stream),
                     "sgd A");
        check_launch(q4::launch_sgd(static_cast<float*>(dB.p), static_cast<float*>(gB.p), learning_rate, 64 * r, c.stream),
                     "sgd B");
        d2h(y, dyo.p, xb, c.stream);
        d2h(a, dA.p, pb, c.stream);
        d2h(b, dB.p, pb, c.stream);
        check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_lora_backward(spaceslug_q4_weights* w, const float* x, const float* dy, uint32_t m,
                                       void* stream) {
    if (!w || !x || !dy || m == 0) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer or m == 0");
    if (w->rank == 0) return fail(SPACESLUG_INVALID_ARGUMENT, "no LoRA adapter attached");
    return guarded([&] {
        check(cudaSetDevice(w->device), "cudaSetDevice");
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        const size_t pa = static_cast<size_t>(w->K) * w->rank * 4, pbb = static_cast<size_t>(w->rank) * w->N * 4;
        if (!w->lora_da) check(cudaMalloc(&w->lora_da, pa), "cudaMalloc dA");
        if (!w->lora_db) check(cudaMalloc(&w->lora_db, pbb), "cudaMalloc dB");
        q4::LoraBackwardArgs g{x, dy, w->lora_a, w->lora_b, w->lora_da, w->lora_db, nullptr,
                               static_cast<int>(m), w->K, w->N, w->rank, w->alpha / static_cast<float>(w->rank)};
        if (lora_backward_tc_suits(g)) {
            DeviceCtx& c = ctx_for(w->device);
            run_lora_backward_tc(g, c.sm_count, c.status, s);
        } else {
            Scratch sc(q4::lora_backward_scratch_floats(static_cast<int>(m), w->K, w->N, w->rank) * 4, s);
            g.scratch = static_cast<float*>(sc.p);
            check_launch(q4::launch_lora_backward(g, s), "lora backward");
        }
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_lora_sgd(spaceslug_q4_weights* w, float learning_rate, void* stream) {
    if (!w || !(learning_rate > 0.0f)) return fail(SPACESLUG_INVALID_ARGUMENT, "null handle or learning_rate <= 0");
    if (!w->lora_da || !w->lora_db) return fail(SPACESLUG_INVALID_ARGUMENT, "no gradients: run the backward first");
    return guarded([&] {
        check(cudaSetDevice(w->device), "cudaSetDevice");
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        check_launch(q4::launch_sgd(w->lora_a, w->lora_da, learning_rate, static_cast<long long>(w->K) * w->rank, s),
                     "sgd A");
        check_launch(q4::launch_sgd(w->lora_b, w->lora_db, learning_rate, static_cast<long long>(w->rank) * w->N, s),
                     "sgd B");
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_lora_adamw(spaceslug_q4_weights* w, float learning_rate, float beta1, float beta2, float eps,
                                    float weight_decay, void* stream) {
    if (!w || !(learning_rate > 0.0f) || !(beta1 >= 0.0f && beta1 < 1.0f) || !(beta2 >= 0.0f && beta2 < 1.0f) ||
        !(eps > 0.0f) || !(weight_decay >= 0.0f))
        return fail(SPACESLUG_INVALID_ARGUMENT, "bad AdamW hyper-parameters");
    if (!w->lora_da || !w->lora_db) return fail(SPACESLUG_INVALID_ARGUMENT, "no gradients: run the backward first");
    return guarded([&] {
        check(cudaSetDevice(w->device), "cudaSetDevice");
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        const long long na = static_cast<long long>(w->K) * w->rank, nb = static_cast<long long>(w->rank) * w->N;
        if (!w->adam) {
            check(cudaMalloc(&w->adam, static_cast<size_t>(2 * (na + nb)) * 4), "cudaMalloc AdamW moments");
            check(cudaMemsetAsync(w->adam, 0, static_cast<size_t>(2 * (na + nb)) * 4, s), "cudaMemset moments");
        }
        ++w->adam_step;
        check_launch(q4::launch_adamw(w->lora_a, w->lora_da, w->adam, w->adam + na, learning_rate, beta1, beta2, eps,
                                      weight_decay, w->adam_step, na, s),
                     "adamw A");
        check_launch(q4::launch_adamw(w->lora_b, w->lora_db, w->adam + 2 * na, w->adam + 2 * na + nb, learning_rate,
                                      beta1, beta2, eps, weight_decay, w->adam_step, nb, s),
                     "adamw B");
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_weights_get_lora(const spaceslug_q4_weights* w, float* a_out, float* b_out, float* da_out,
                                  float* db_out) {
    if (!w) return fail(SPACESLUG_INVALID_ARGUMENT, "null handle");
    if (w->rank == 0) return fail(SPACESLUG_INVALID_ARGUMENT, "no LoRA adapter attached");
    if ((da_out || db_out) && (!w->lora_da || !w->lora_db))
        return fail(SPACESLUG_INVALID_ARGUMENT, "no gradients: run the backward first");
    return guarded([&] {
        check(cudaSetDevice(w->device), "cudaSetDevice");
        check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
        const size_t pa = static_cast<size_t>(w->K) * w->rank * 4, pbb = static_cast<size_t>(w->rank) * w->N * 4;
        if (a_out) check(cudaMemcpy(a_out, w->lora_a, pa, cudaMemcpyDeviceToHost), "D2H A");
        if (b_out) check(cudaMemcpy(b_out, w->lora_b, pbb, cudaMemcpyDeviceToHost), "D2H B");
        if (da_out) check(cudaMemcpy(da_out, w->lora_da, pa, cudaMemcpyDeviceToHost), "D2H dA");
        if (db_out) check(cudaMemcpy(db_out, w->lora_db, pbb, cudaMemcpyDeviceToHost), "D2H dB");
        return SPACESLUG_OK;
    });
}

int spaceslug_q4_set_operand_type(int type) {
    if (type != 0 && type != 1) return -1;
    operand_type();  // apply the environment default first
    return g_operand.exchange(type);
}

int spaceslug_q4_set_decode_variant(int variant) {
    if (variant < 0 || variant > 4) return -1;
    return decode_variant_init().exchange(variant);
}

int spaceslug_q4_set_gemm_variant(int variant) {
    if (variant < 0 || variant > 3) return -1;
    return g_gemm_variant.exchange(variant);
}

int spaceslug_q4_device_status(int device) {
    if (device < 0 || device >= kMaxDevices) return fail(SPACESLUG_INVALID_ARGUMENT, "device ordinal out of range");
    return guarded([&] {
        check(cudaSetDevice(device), "cudaSetDevice");
        check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
        // The context's word exists only once a regular entry point ran on the
        // device; this call does not create the context (it allocates), so a
        // caller of the no-allocation entry point alone allocates nothing here.
        int st = 0;
        DeviceCtx& c = g_ctx[device];
        if (c.ready.load(std::memory_order_acquire)) {
            check(cudaMemcpy(&st, c.status, sizeof(int), cudaMemcpyDeviceToHost), "read status");
            if (st) check(cudaMemset(c.status, 0, sizeof(int)), "clear status");
        }
        int st_noalloc = 0;
        check(q4rt::noalloc_take_status(device, &st_noalloc), "read the no-allocation status word");
        return st != 0 ? st : st_noalloc;
    });
}

int spaceslug_q4_debug_wait_test(uint64_t wait_limit_ns, int stall) {
    return guarded([&] {
        const unsigned long long lim = wait_limit_ns ? wait_limit_ns : 2000000000ull;
        const int st = stall ? 1 : 0;
        check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");  // no launch in flight sees a half-set hook
        check(static_cast<cudaError_t>(q4::gemv_tile_set_wait_test(lim, st)), "set the tile GEMV test hook");
        check(static_cast<cudaError_t>(q4::gemv_ring_set_wait_test(lim, st)), "set the ring GEMV test hook");
        check(static_cast<cudaError_t>(q4::gemv_imma_set_wait_test(lim, st)), "set the IMMA GEMV test hook");
        return SPACESLUG_OK;
    });
}

uint64_t spaceslug_q4_launch_count(void) { return g_launches.load(); }

const char* spaceslug_last_error(void) { return g_last_error.c_str(); }

int spaceslug_sgemm(const float* a, const float* b, float* c, uint32_t m, uint32_t n, uint32_t k,
                    float* max_relative_error) {
    // Same checks as vulkan-runtime/src/api/sgemm_api.cpp:25.
    if (!a || !b || !c || !max_relative_error || m == 0 || n == 0 || k == 0 || m % 64 || n % 64 || k % 32)
        return fail(SPACESLUG_INVALID_ARGUMENT, "need non-null pointers, M, N % 64 == 0 and K % 32 == 0");
    return guarded([&] {
        DeviceCtx& ctx = ctx_for(current_device());
        std::lock_guard<std::mutex> lk(ctx.host_mu);
        const size_t ab = static_cast<size_t>(m) * k * 4, bb = static_cast<size_t>(k) * n * 4,
                     cb = static_cast<size_t>(m) * n * 4;
        Scratch da(ab, ctx.stream), db(bb, ctx.stream), dc(cb, ctx.stream);
        q4up::staged_h2d(current_device(), da.p, a, ab, ctx.stream);
        q4up::staged_h2d(current_device(), db.p, b, bb, ctx.stream);
        run_sgemm(static_cast<float*>(da.p), k, false, static_cast<float*>(db.p), n, false, static_cast<float*>(dc.p),
                  n, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), 1.0f, ctx.status, ctx.stream);
        d2h(c, dc.p, cb, ctx.stream);
        if (take_status(ctx, ctx.stream)) return fail(SPACESLUG_TIMEOUT, "a kernel wait timed out");
        *max_relative_error = 0.0f;  // the reference reports 0 as well (sgemm_api.cpp:54)
        return SPACESLUG_OK;
    });
}

int spaceslug_sgemm_device(const float* a, const float* b, float* c, uint32_t m, uint32_t n, uint32_t k, void* stream) {
    if (!a || !b || !c || m == 0 || n == 0 || k == 0) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer or zero dimension");
    if (m > (1u << 30) || n > (1u << 30) || k > (1u << 30)) return fail(SPACESLUG_INVALID_ARGUMENT, "dimension too large");
    return guarded([&] {
        DeviceCtx& ctx = ctx_for(current_device());
        run_sgemm(a, k, false, b, n, false, c, n, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), 1.0f,
                  ctx.status, static_cast<cudaStream_t>(stream));
        return SPACESLUG_OK;
    });
}

int spaceslug_shards_relayout(const float* gathered, float* y, uint32_t parts, uint32_t rows, uint32_t width,
                              uint32_t n_total, uint64_t ld_y, void* stream) {
    if (!gathered || !y) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (parts == 0 || width == 0 || n_total == 0) return fail(SPACESLUG_INVALID_ARGUMENT, "zero dimension");
    if (parts > (1u << 16) || rows > (1u << 30) || width > (1u << 30))
        return fail(SPACESLUG_INVALID_ARGUMENT, "dimension too large");
    if (static_cast<uint64_t>(n_total) > static_cast<uint64_t>(parts) * width)
        return fail(SPACESLUG_INVALID_ARGUMENT, "n_total exceeds parts * width");
    if (ld_y < n_total || ld_y > (uint64_t(1) << 40)) return fail(SPACESLUG_INVALID_ARGUMENT, "bad ld_y");
    if (rows == 0) return SPACESLUG_OK;
    return guarded([&] {
        check_launch(q4::launch_shards_relayout(gathered, y, static_cast<int>(parts), static_cast<int>(rows),
                                                static_cast<int>(width), static_cast<int>(n_total),
                                                static_cast<long long>(ld_y), static_cast<cudaStream_t>(stream)),
                     "shards_relayout");
        return SPACESLUG_OK;
    });
}

int spaceslug_cq4_weights_create(const spaceslug_cq4_matrix* m, int device, spaceslug_cq4_weights** out) {
    if (!m || !out) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    *out = nullptr;
    if (m->bits != 4) return fail(SPACESLUG_INVALID_ARGUMENT, "only 4-bit CQ4 indices are supported");
    if (!m->codebook || !m->norms || !m->packed_indices) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (m->k == 0 || m->n == 0 || m->k % 32u) return fail(SPACESLUG_INVALID_ARGUMENT, "K must be a positive multiple of 32");
    const bool orth = (m->flags & SPACESLUG_CQ4_FLAG_ORTHOGONAL) != 0;
    const bool il = (m->flags & SPACESLUG_CQ4_FLAG_INTERLEAVED_4ROW) != 0;
    if (il && m->n % 4u) return fail(SPACESLUG_INVALID_ARGUMENT, "INTERLEAVED_4ROW needs N % 4 == 0");
    if (orth) {
        if (!m->rotation) return fail(SPACESLUG_INVALID_ARGUMENT, "orthogonal mode needs the rotation");
    } else {
        const uint32_t gs = m->group_size;
        if (gs < 32 || gs > 256 || (gs & (gs - 1))) return fail(SPACESLUG_INVALID_ARGUMENT, "group_size must be 32, 64, 128 or 256");
        if (m->num_groups == 0 || gs * m->num_groups != m->k) return fail(SPACESLUG_INVALID_ARGUMENT, "K != group_size * num_groups");
        if (m->permutation)
            for (uint32_t j = 0; j < gs; ++j)
                if (m->permutation[j] >= gs) return fail(SPACESLUG_INVALID_ARGUMENT, "permutation entry out of range");
    }
    return guarded([&] {
        check(cudaSetDevice(device), "cudaSetDevice");
        DeviceCtx& c = ctx_for(device);
        const uint32_t K = m->k, N = m->n, gs = orth ? K : m->group_size;
        // host preparation
        std::vector<uint8_t> packed(static_cast<size_t>(N) * K / 2, 0);
        if (il) {
            for (uint32_t n = 0; n < N; ++n)
                for (uint32_t k = 0; k < K; k += 2)
                    packed[static_cast<size_t>(n) * K / 2 + k / 2] =
                        static_cast<uint8_t>(cq4_index(*m, orth, n, k) | (cq4_index(*m, orth, n, k + 1) << 4));
        } else {
            std::memcpy(packed.data(), m->packed_indices, packed.size());  // already [N][K/2], low nibble = even k
        }
        std::vector<float> scales(static_cast<size_t>(N) * (K / 32));
        for (uint32_t n = 0; n < N; ++n)
            for (uint32_t j = 0; j < K / 32; ++j)
                scales[static_cast<size_t>(n) * (K / 32) + j] = cq4_norm(*m, orth, n, orth ? 0u : (32u * j) / gs);
        std::vector<uint32_t> lut(256);
        for (uint32_t b = 0; b < 256; ++b)
            lut[b] = static_cast<uint32_t>(m->codebook[b & 15u]) | (static_cast<uint32_t>(m->codebook[b >> 4]) << 16);
        std::vector<float> recip(K, 1.0f);
        for (uint32_t k = 0; k < K; ++k) {
            if (m->input_scale_recip) recip[k] = half_bits_to_float(m->input_scale_recip[k]);
            else if (m->input_scale) recip[k] = 1.0f / half_bits_to_float(m->input_scale[k]);
        }
        auto* w = new spaceslug_cq4_weights();
        w->device = device;
        w->K = static_cast<int>(K);
        w->N = static_cast<int>(N);
        w->gs = static_cast<int>(gs);
        w->orthogonal = orth;
        w->inv_sqrt = 1.0f / std::sqrt(static_cast<float>(gs));
        try {
            std::lock_guard<std::mutex> lk(c.host_mu);
            auto upload = [&](auto** dst, const void* src, size_t bytes) {
                check(cudaMalloc(reinterpret_cast<void**>(dst), bytes), "cudaMalloc cq4");
                q4up::staged_h2d(device, *dst, src, bytes, c.stream);
            };
            upload(&w->packed, packed.data(), packed.size());
            upload(&w->scales, scales.data(), scales.size() * 4);
            upload(&w->lut, lut.data(), lut.size() * 4);
            float cbf[16];
            for (int i = 0; i < 16; ++i) cbf[i] = half_bits_to_float(m->codebook[i]);
            upload(&w->cbf, cbf, sizeof(cbf));
            upload(&w->recip, recip.data(), recip.size() * 4);
            if (!orth) {
                std::vector<float> sg(gs);
                if (m->left_signs) {
                    for (uint32_t j = 0; j < gs; ++j) sg[j] = static_cast<float>(m->left_signs[j]);
                    upload(&w->lsign, sg.data(), gs * 4);
                }
                if (m->right_signs) {
                    for (uint32_t j = 0; j < gs; ++j) sg[j] = static_cast<float>(m->right_signs[j]);
                    upload(&w->rsign, sg.data(), gs * 4);
                }
                if (m->permutation) upload(&w->perm, m->permutation, gs * 4);
            } else {
                upload(&w->rotation, m->rotation, static_cast<size_t>(K) * K * 2);
            }
            check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        } catch (...) {
            spaceslug_cq4_weights_destroy(w);
            throw;
        }
        *out = w;
        return SPACESLUG_OK;
    });
}

int spaceslug_cq4_matmul(spaceslug_cq4_weights* w, const uint16_t* a, uint16_t* c, uint32_t m, void* stream) {
    if (!w || !a || !c || m == 0) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer or m == 0");
    if (m > (1u << 30)) return fail(SPACESLUG_INVALID_ARGUMENT, "m too large");
    return guarded([&] {
        check(cudaSetDevice(w->device), "cudaSetDevice");
        run_cq4(*w, a, c, static_cast<int>(m), static_cast<cudaStream_t>(stream));
        return SPACESLUG_OK;
    });
}

int spaceslug_cq4_matmul_host(spaceslug_cq4_weights* w, const uint16_t* a, uint16_t* c, uint32_t m) {
    if (!w || !a || !c || m == 0) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer or m == 0");
    return guarded([&] {
        check(cudaSetDevice(w->device), "cudaSetDevice");
        DeviceCtx& ctx = ctx_for(w->device);
        std::lock_guard<std::mutex> lk(ctx.host_mu);
        const size_t ab = static_cast<size_t>(m) * w->K * 2, cb = static_cast<size_t>(m) * w->N * 2;
        Scratch da(ab, ctx.stream), dc(cb, ctx.stream);
        h2d(da.p, a, ab, ctx.stream);
        run_cq4(*w, da.p, dc.p, static_cast<int>(m), ctx.stream);
        d2h(c, dc.p, cb, ctx.stream);
        check(cudaStreamSynchronize(ctx.stream), "cudaStreamSynchronize");
        if (take_status(ctx, ctx.stream)) return fail(SPACESLUG_TIMEOUT, "a kernel wait timed out");
        return SPACESLUG_OK;
    });
}

int spaceslug_cq4_transform_host(spaceslug_cq4_weights* w, const uint16_t* a, uint16_t* a_out, uint32_t m) {
    if (!w || !a || !a_out || m == 0) return fail(SPACESLUG_INVALID_ARGUMENT, "null pointer or m == 0");
    return guarded([&] {
        check(cudaSetDevice(w->device), "cudaSetDevice");
        DeviceCtx& ctx = ctx_for(w->device);
        std::lock_guard<std::mutex> lk(ctx.host_mu);
        const size_t ab = static_cast<size_t>(m) * w->K * 2;
        Scratch da(ab, ctx.stream), dout(ab, ctx.stream);
        h2d(da.p, a, ab, ctx.stream);
        check_launch(q4::launch_cq4_transform(da.p, dout.p, w->recip, w->lsign, w->rsign, w->perm, w->rotation,
                                              static_cast<int>(m), w->K, w->gs, w->inv_sqrt, ctx.stream),
                     "cq4 transform");
        d2h(a_out, dout.p, ab, ctx.stream);
        check(cudaStreamSynchronize(ctx.stream), "cudaStreamSynchronize");
        return SPACESLUG_OK;
    });
}

int spaceslug_cq4_weights_destroy(spaceslug_cq4_weights* w) {
    if (!w) return fail(SPACESLUG_INVALID_ARGUMENT, "null handle");
    cudaSetDevice(w->device);
    for (void* p : {static_cast<void*>(w->packed), static_cast<void*>(w->scales), static_cast<void*>(w->lut),
                    static_cast<void*>(w->cbf),
                    static_cast<void*>(w->recip), static_cast<void*>(w->lsign), static_cast<void*>(w->rsign),
                    static_cast<void*>(w->perm), static_cast<void*>(w->rotation)})
        cudaFree(p);
    delete w;
    return SPACESLUG_OK;
}

}  // extern "C"
