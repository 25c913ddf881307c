// Model-load path of the int4 weights: the reference packs on one CPU core
// (vulkan-runtime/tests/test_q4gemm.cpp:84-99) and copies from pageable
// memory.  Here the host packer runs on several threads, uploads go through a
// per-device ring of pinned slots (several host threads fill slot i + 1 while
// the DMA engine drains slot i), and the packing itself can run on the device
// from the logical int8 matrix, which then only has to cross PCIe as bytes.
// Measured on the B200 hosts (16 CPUs, one NUMA node): a host memcpy reaches
// ~55 GB/s with 4-8 threads and a pinned H2D copy ~55 GB/s, so 8-MiB slots
// filled by 8 threads of a persistent pool keep both busy (spawning the
// threads per slot cost more than the copies).
#include <cuda_runtime.h>
#include <sched.h>

#include <algorithm>
#include <array>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "upload.h"

namespace q4up {

namespace {

constexpr int kSlots = 4;
constexpr size_t kSlotBytes = size_t(8) << 20;  // 8 MiB per pinned slot
constexpr int kCopyThreads = 8;                 // threads per staging copy
constexpr size_t kDirectBytes = size_t(1) << 20; // below this a plain copy is cheaper than staging
constexpr int kMaxDevices = 64;

void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Host threads for the staging copies and the packer: the CPUs this process
// may run on (its affinity mask, which a container's CPU set narrows; not the
// machine's core count), at most 16.
int copy_threads() {
    static const int n = [] {
        cpu_set_t set;
        CPU_ZERO(&set);
        int c = 0;
        if (sched_getaffinity(0, sizeof(set), &set) == 0) c = CPU_COUNT(&set);
        if (c <= 0) c = static_cast<int>(std::thread::hardware_concurrency());
        return std::max(1, std::min(16, c));
    }();
    return n;
}

// Persistent host worker threads (copy_threads() - 1 of them besides the
// caller), created on first use.  run(parts, f) calls f(i) for i in
// [0, parts): thread t (0 = the caller) takes parts t, t + T, ... (T threads
// in all) and run returns when every part is done.  One job at a time.
class WorkerPool {
public:
    static WorkerPool& get() {
        static WorkerPool pool(copy_threads() - 1);
        return pool;
    }
    int threads() const { return static_cast<int>(workers_.size()) + 1; }
    void run(int parts, const std::function<void(int)>& f) {
        std::lock_guard<std::mutex> job_lock(job_mu_);
        const int T = threads();
        if (parts <= 1 || T == 1) {
            for (int i = 0; i < parts; ++i) f(i);
            return;
        }
        {
            std::lock_guard<std::mutex> lk(mu_);
            job_ = &f;
            parts_ = parts;
            pending_ = T - 1;
            ++generation_;
        }
        cv_.notify_all();
        for (int i = 0; i < parts; i += T) f(i);
        std::unique_lock<std::mutex> lk(mu_);
        done_cv_.wait(lk, [&] { return pending_ == 0; });
        job_ = nullptr;
    }
    ~WorkerPool() {
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto& t : workers_) t.join();
    }

private:
    explicit WorkerPool(int n) {
        for (int w = 1; w <= n; ++w)
            workers_.emplace_back([this, w] {
                unsigned long long seen = 0;
                for (;;) {
                    const std::function<void(int)>* f;
                    int parts, T;
                    {
                        std::unique_lock<std::mutex> lk(mu_);
                        cv_.wait(lk, [&] { return stop_ || generation_ != seen; });
                        if (stop_) return;
                        seen = generation_;
                        f = job_;
                        parts = parts_;
                        T = threads();
                    }
                    for (int i = w; i < parts; i += T) (*f)(i);
                    std::lock_guard<std::mutex> lk(mu_);
                    if (--pending_ == 0) done_cv_.notify_one();
                }
            });
    }
    std::vector<std::thread> workers_;
    std::mutex job_mu_, mu_;
    std::condition_variable cv_, done_cv_;
    const std::function<void(int)>* job_ = nullptr;
    int parts_ = 0, pending_ = 0;
    unsigned long long generation_ = 0;
    bool stop_ = false;
};

// Runs f(i) for i in [0, parts) on the worker pool.
template <typename F>
void parallel_for(int parts, F&& f) {
    const std::function<void(int)> job(std::forward<F>(f));
    WorkerPool::get().run(parts, job);
}

void parallel_memcpy(void* dst, const void* src, size_t bytes) {
    const int parts = bytes >= (size_t(1) << 20) ? std::min(kCopyThreads, copy_threads()) : 1;
    const size_t per = (bytes + parts - 1) / parts;
    parallel_for(parts, [&](int i) {
        const size_t b = i * per;
        if (b < bytes) std::memcpy(static_cast<char*>(dst) + b, static_cast<const char*>(src) + b, std::min(per, bytes - b));
    });
}

// rows x ncols bytes from a row-major matrix with row pitch `pitch` into a
// dense block.
void parallel_rows_copy(int8_t* dst, const int8_t* src, size_t rows, size_t ncols, size_t pitch) {
    const int parts = rows * ncols >= (size_t(1) << 20) ? std::min(kCopyThreads, copy_threads()) : 1;
    const size_t per = (rows + parts - 1) / parts;
    parallel_for(parts, [&](int i) {
        const size_t r0 = i * per, r1 = std::min(rows, r0 + per);
        for (size_t r = r0; r < r1; ++r) std::memcpy(dst + r * ncols, src + r * pitch, ncols);
    });
}

struct Ring {
    std::mutex mu;
    bool ready = false;
    std::array<void*, kSlots> host{};
    std::array<cudaEvent_t, kSlots> done{};
};
Ring g_rings[kMaxDevices];

Ring& ring_for(int device) {
    if (device < 0 || device >= kMaxDevices) throw std::runtime_error("device ordinal out of range");
    return g_rings[device];
}

// Called with r.mu held and `device` current.
void ring_init(Ring& r) {
    if (r.ready) return;
    for (int i = 0; i < kSlots; ++i) {
        ck(cudaHostAlloc(&r.host[i], kSlotBytes, cudaHostAllocDefault), "cudaHostAlloc staging slot");
        ck(cudaEventCreateWithFlags(&r.done[i], cudaEventDisableTiming), "cudaEventCreate");
    }
    r.ready = true;
}

bool is_pinned(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();  // a plain pageable pointer on older drivers
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

// Chunk c of the logical int8 block [rows][ncols] -> packed words: thread
// (column n, quad q) builds 4 consecutive words (32 rows) of column n with
// coalesced byte reads across the warp and writes them as one 16-byte store.
__global__ void __launch_bounds__(256) pack_rows_kernel(const int8_t* __restrict__ blk, uint32_t* __restrict__ packed,
                                                        int rows, int ncols, int c0, int chunks_total) {
    const int quads = (rows / 8 + 3) / 4;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(ncols) * quads) return;
    const int n = static_cast<int>(idx % ncols), qd = static_cast<int>(idx / ncols);
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int c = qd * 4 + j;
        uint32_t word = 0;
        if (c * 8 < rows) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                word |= (static_cast<uint32_t>(static_cast<uint8_t>(blk[static_cast<size_t>(c * 8 + i) * ncols + n])) & 0xFu)
                        << (4 * i);
        }
        w[j] = word;
    }
    uint32_t* out = packed + static_cast<size_t>(n) * chunks_total + c0 + qd * 4;
    const int left = rows / 8 - qd * 4;
    if (left >= 4 && ((reinterpret_cast<uintptr_t>(out) & 15u) == 0)) {
        *reinterpret_cast<uint4*>(out) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        for (int j = 0; j < 4 && j < left; ++j) out[j] = w[j];
    }
}

}  // namespace

void host_pack(const int8_t* w_kn, uint32_t k, uint32_t n, uint32_t* packed_out, int threads) {
    const uint32_t chunks = k / 8u;
    const int parts = std::max(1, std::min<int>(threads > 0 ? threads : copy_threads(), static_cast<int>(chunks)));
    const uint32_t per = (chunks + parts - 1) / parts;
    parallel_for(parts, [&](int p) {
        // each thread owns chunks [c0, c1): 8 source rows per output word, the
        // words of one chunk assembled in a row-sized register file
        const uint32_t c0 = p * per, c1 = std::min(chunks, c0 + per);
        std::vector<uint32_t> acc(n);
        for (uint32_t c = c0; c < c1; ++c) {
            std::fill(acc.begin(), acc.end(), 0u);
            for (uint32_t i = 0; i < 8u; ++i) {
                const int8_t* row = w_kn + static_cast<size_t>(8u * c + i) * n;
                const uint32_t shift = 4u * i;
                for (uint32_t col = 0; col < n; ++col)
                    acc[col] |= (static_cast<uint32_t>(static_cast<uint8_t>(row[col])) & 0xFu) << shift;
            }
            for (uint32_t col = 0; col < n; ++col) packed_out[static_cast<size_t>(col) * chunks + c] = acc[col];
        }
    });
}

void staged_h2d(int device, void* dst, const void* src, size_t bytes, cudaStream_t stream) {
    if (bytes == 0) return;
    if (bytes < kDirectBytes || is_pinned(src)) {
        ck(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream), "cudaMemcpyAsync H2D");
        if (bytes < kDirectBytes) ck(cudaStreamSynchronize(stream), "cudaStreamSynchronize");  // src may be pageable
        return;
    }
    Ring& r = ring_for(device);
    std::lock_guard<std::mutex> lk(r.mu);
    ring_init(r);
    size_t off = 0;
    for (int i = 0; off < bytes; ++i) {
        const size_t len = std::min(kSlotBytes, bytes - off);
        const int s = i % kSlots;
        ck(cudaEventSynchronize(r.done[s]), "staging slot wait");
        parallel_memcpy(r.host[s], static_cast<const char*>(src) + off, len);
        ck(cudaMemcpyAsync(static_cast<char*>(dst) + off, r.host[s], len, cudaMemcpyHostToDevice, stream),
           "cudaMemcpyAsync H2D (staged)");
        ck(cudaEventRecord(r.done[s], stream), "cudaEventRecord");
        off += len;
    }
}

void staged_pack_logical(int device, uint32_t* packed_dev, const int8_t* w_kn, uint32_t k, uint32_t n_total,
                         uint32_t col_begin, uint32_t ncols, cudaStream_t stream) {
    if (static_cast<size_t>(ncols) * 32 > kSlotBytes) throw std::runtime_error("too many columns for one staging slot");
    // rows per block: a multiple of 32 (whole 16-byte packed quads) that fits a slot
    size_t rows_blk = kSlotBytes / ncols / 32 * 32;
    rows_blk = std::min<size_t>(rows_blk, k);
    Ring& r = ring_for(device);
    std::lock_guard<std::mutex> lk(r.mu);
    ring_init(r);
    std::array<void*, kSlots> dev{};
    try {
        for (int i = 0; i < kSlots; ++i)
            ck(cudaMallocAsync(&dev[i], rows_blk * ncols, stream), "cudaMallocAsync pack staging");
        const int chunks_total = static_cast<int>(k / 8u);
        int i = 0;
        for (size_t k0 = 0; k0 < k; k0 += rows_blk, ++i) {
            const size_t rows = std::min<size_t>(rows_blk, k - k0);
            const int s = i % kSlots;
            ck(cudaEventSynchronize(r.done[s]), "staging slot wait");
            parallel_rows_copy(static_cast<int8_t*>(r.host[s]), w_kn + k0 * n_total + col_begin, rows, ncols, n_total);
            ck(cudaMemcpyAsync(dev[s], r.host[s], rows * ncols, cudaMemcpyHostToDevice, stream),
               "cudaMemcpyAsync H2D (logical)");
            const long long work = static_cast<long long>(ncols) * ((rows / 8 + 3) / 4);
            pack_rows_kernel<<<static_cast<unsigned>((work + 255) / 256), 256, 0, stream>>>(
                static_cast<const int8_t*>(dev[s]), packed_dev, static_cast<int>(rows), static_cast<int>(ncols),
                static_cast<int>(k0 / 8), chunks_total);
            ck(cudaGetLastError(), "pack_rows launch");
            ck(cudaEventRecord(r.done[s], stream), "cudaEventRecord");
        }
    } catch (...) {
        for (void* p : dev)
            if (p) cudaFreeAsync(p, stream);
        throw;
    }
    for (void* p : dev) ck(cudaFreeAsync(p, stream), "cudaFreeAsync pack staging");
}

}  // namespace q4up
