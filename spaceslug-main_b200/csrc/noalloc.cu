// spaceslug_q4gemv_lora_noalloc: the decode GEMV with the fused LoRA term for
// callers that cannot allocate device memory.
//
// Some callers of this library may not call cudaMalloc (or the stream-ordered
// cudaMallocAsync the regular entry points use for scratch): a serving loop
// that forbids allocation on its hot path (an allocation can stall or
// synchronise the device), or a plugin host that has reserved all device
// memory for itself and hands the plugin only its input and output buffers.  This entry point keeps its only scratch, the LoRA projection
// T = X * A (at most kMaxRows x kMaxRank floats = 2 KB), in a file-scope
// static __device__ array, so a call allocates nothing.
//
// The array exists once per GPU that loads the library and stays there until
// the process exits.  Every call on a device uses the same array and leaves
// the last call's T in it; each call writes all of T that it reads, so nothing
// needs clearing, but two calls that overlap on the GPU (different streams,
// or different host threads) race on it and must be ordered by the caller.
//
// Host code cannot take the array's address directly: in host code the
// symbol names a host-side stand-in.  The first call on each device, with that
// device current, looks up the device address with cudaGetSymbolAddress
// (and the kernels load); make that first call before any stream capture.
//
// A kernel wait that runs out of time (the kernels bound every wait) records
// a code in a second static word, g_noalloc_status; the call itself is
// asynchronous and returns before the kernel runs, so the caller learns of a
// timeout from spaceslug_q4_device_status(device), which reads and clears
// this word (with cudaMemcpyFromSymbol / cudaMemcpyToSymbol: no allocation).
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdint>
#include <mutex>

#include "../../include/runtime_abi.h"
#include "q4_kernels.h"

namespace q4rt {
bool gemv_geometry(int sm_count, int M, int N, int K, int* S, int* clusters, int* cols);
bool encode_gemv_weights(CUtensorMap* map, const uint32_t* packed, int N, int K, int S);
void count_launch();
int set_error(int code, const char* msg);
}  // namespace q4rt

namespace {

constexpr int kMaxRows = 8;   // decode rows (M)
constexpr int kMaxRank = 64;  // LoRA rank

static __device__ __align__(256) float g_lora_t_scratch[kMaxRows * kMaxRank];
static __device__ __align__(256) int g_noalloc_status;  // kernel wait-timeout word

struct DeviceState {
    std::once_flag once;
    std::atomic<bool> ready{false};  // set once the symbol addresses are known
    cudaError_t err = cudaSuccess;
    float* t = nullptr;
    int* status = nullptr;
    int sm_count = 0;
};
constexpr int kMaxDevices = 64;
DeviceState g_state[kMaxDevices];

}  // namespace

namespace q4rt {
// Reads and clears the status word of the no-allocation entry point on
// `device` (the current device; the caller has synchronised it).  *out is 0
// when that entry point never ran there.
cudaError_t noalloc_take_status(int device, int* out) {
    *out = 0;
    if (device < 0 || device >= kMaxDevices || !g_state[device].ready.load(std::memory_order_acquire))
        return cudaSuccess;
    cudaError_t e = cudaMemcpyFromSymbol(out, g_noalloc_status, sizeof(int));
    if (e == cudaSuccess && *out != 0) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_noalloc_status, &zero, sizeof(int));
    }
    return e;
}
}  // namespace q4rt

extern "C" int spaceslug_q4gemv_lora_noalloc(const float* x, const uint32_t* packed, const float* scales,
                                             const float* lora_a, const float* lora_b, uint32_t rank, float alpha,
                                             float* y, uint32_t m, uint32_t n, uint32_t k, void* stream) {
    if (!x || !packed || !scales || !lora_a || !lora_b || !y)
        return q4rt::set_error(SPACESLUG_INVALID_ARGUMENT, "null pointer");
    if (m == 0 || m > static_cast<uint32_t>(kMaxRows))
        return q4rt::set_error(SPACESLUG_INVALID_ARGUMENT, "m must be 1..8 for the no-allocation entry point");
    if (rank == 0 || rank > static_cast<uint32_t>(kMaxRank))
        return q4rt::set_error(SPACESLUG_INVALID_ARGUMENT, "rank must be 1..64 for the no-allocation entry point");
    if (n == 0 || k == 0 || k % 32u || n > (1u << 30) || k > (1u << 30))
        return q4rt::set_error(SPACESLUG_INVALID_ARGUMENT, "k must be a positive multiple of 32, n > 0");
    if (!std::isfinite(alpha)) return q4rt::set_error(SPACESLUG_INVALID_ARGUMENT, "alpha must be finite");
    const auto mis16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; };
    if (mis16(x) || mis16(packed) || mis16(y))
        return q4rt::set_error(SPACESLUG_INVALID_ARGUMENT, "x, packed and y must be 16-byte aligned");

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return q4rt::set_error(SPACESLUG_RUNTIME_FAILURE, "no current CUDA device");
    DeviceState& st = g_state[dev];
    std::call_once(st.once, [&] {
        void* p = nullptr;
        st.err = cudaGetSymbolAddress(&p, g_lora_t_scratch);
        if (st.err != cudaSuccess) return;
        st.t = static_cast<float*>(p);
        st.err = cudaGetSymbolAddress(&p, g_noalloc_status);
        if (st.err != cudaSuccess) return;
        st.status = static_cast<int*>(p);
        st.err = cudaDeviceGetAttribute(&st.sm_count, cudaDevAttrMultiProcessorCount, dev);
        if (st.err == cudaSuccess) st.ready.store(true, std::memory_order_release);
    });
    if (st.err != cudaSuccess) return q4rt::set_error(SPACESLUG_RUNTIME_FAILURE, cudaGetErrorString(st.err));

    int S = 0, clusters = 0, cols = 0;
    if (!q4rt::gemv_geometry(st.sm_count, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), &S,
                             &clusters, &cols))
        return q4rt::set_error(SPACESLUG_INVALID_ARGUMENT,
                               "shape not supported by the no-allocation entry point (K/32 must split into at most "
                               "8 slices of at most 32 scale groups)");
    q4::GemvArgs a{};
    if (!q4rt::encode_gemv_weights(&a.tmap_w, packed, static_cast<int>(n), static_cast<int>(k), S))
        return q4rt::set_error(SPACESLUG_RUNTIME_FAILURE, "tensor map encoding failed");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int e = q4::launch_lora_xa(x, lora_a, st.t, static_cast<int>(m), static_cast<int>(k), static_cast<int>(rank), s);
    if (e != 0) return q4rt::set_error(SPACESLUG_RUNTIME_FAILURE, cudaGetErrorString(static_cast<cudaError_t>(e)));
    q4rt::count_launch();
    a.x = x;
    a.scales = scales;
    a.y = y;
    a.M = static_cast<int>(m);
    a.N = static_cast<int>(n);
    a.K = static_cast<int>(k);
    a.cluster_k = S;
    a.clusters = clusters;
    a.cols_per_cluster = cols;
    a.lora_t = st.t;
    a.lora_b = lora_b;
    a.rank = static_cast<int>(rank);
    a.lora_scale = alpha / static_cast<float>(rank);
    a.status = st.status;
    e = q4::launch_gemv(a, s);
    if (e != 0) return q4rt::set_error(SPACESLUG_RUNTIME_FAILURE, cudaGetErrorString(static_cast<cudaError_t>(e)));
    q4rt::count_launch();
    return SPACESLUG_OK;
}
