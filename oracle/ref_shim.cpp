// C-ABI wrapper around the reference's own CPU oracle functions.
//
// TEST INFRASTRUCTURE ONLY (the shipped library never loads it).  The
// reference code itself is NOT in this repository: oracle/Makefile extracts
// vulkan-runtime/tests/test_q4gemm.cpp:57-119 (generate_floats, generate_int4,
// pack_q4, cpu_reference) from the read-only reference checkout into the
// git-ignored oracle/_ref/q4_ref_body.inc at build time, and this file
// compiles it unmodified inside a namespace.  The built library
// oracle/_ref/libq4ref.so is used (a) to pin the C restatement in
// oracle/q4_oracle.c and to generate tests/golden/ fixtures, and (b) as the
// timed CPU baseline ("kind": "reference") of bench.py.
#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace spaceslug_reference {
#include "q4_ref_body.inc"
}  // namespace spaceslug_reference

namespace ref = spaceslug_reference;

namespace {
// One prepared reference problem: the reference function takes std::vector
// arguments, so inputs are copied into vectors once, outside any timing.
struct Problem {
    std::vector<float> a;
    std::vector<std::int8_t> b;
    std::vector<float> scales;
    std::uint32_t m = 0, n = 0, k = 0;
    std::vector<double> c;
};
}  // namespace

extern "C" {

void ref_generate_floats(std::size_t n, std::uint32_t seed, float lo, float hi, float* out) {
    auto v = ref::generate_floats(n, seed, lo, hi);
    std::copy(v.begin(), v.end(), out);
}

void ref_generate_int4(std::size_t n, std::uint32_t seed, std::int8_t* out) {
    auto v = ref::generate_int4(n, seed);
    std::copy(v.begin(), v.end(), out);
}

// packed_out must hold K*N/8 words.
void ref_pack_q4(const std::int8_t* b_kn, std::uint32_t k, std::uint32_t n, std::uint32_t* packed_out) {
    std::vector<std::int8_t> b(b_kn, b_kn + static_cast<std::size_t>(k) * n);
    auto p = ref::pack_q4(b, k, n);
    std::copy(p.begin(), p.end(), packed_out);
}

void ref_cpu_reference(const float* a, const std::int8_t* b_kn, const float* scales,
                       std::uint32_t m, std::uint32_t n, std::uint32_t k, double* c_out) {
    std::vector<float> av(a, a + static_cast<std::size_t>(m) * k);
    std::vector<std::int8_t> bv(b_kn, b_kn + static_cast<std::size_t>(k) * n);
    std::vector<float> sv(scales, scales + static_cast<std::size_t>(n) * (k / 32u));
    auto c = ref::cpu_reference(av, bv, sv, m, n, k);
    std::copy(c.begin(), c.end(), c_out);
}

// Prepared problems for timing: split the N columns of one problem into
// `parts` independent column shards (each a complete reference problem with
// its own K x N_p int8 matrix and its contiguous scale rows), so that the
// unmodified reference function can run on several host threads.
void* ref_prepare(const float* a, const std::int8_t* b_kn, const float* scales,
                  std::uint32_t m, std::uint32_t n, std::uint32_t k, std::uint32_t parts) {
    if (parts == 0 || n % parts != 0 || k % 32u != 0) return nullptr;
    const std::uint32_t np = n / parts, groups = k / 32u;
    auto* ps = new std::vector<Problem>(parts);
    for (std::uint32_t p = 0; p < parts; ++p) {
        Problem& pr = (*ps)[p];
        pr.m = m; pr.n = np; pr.k = k;
        pr.a.assign(a, a + static_cast<std::size_t>(m) * k);
        pr.b.resize(static_cast<std::size_t>(k) * np);
        for (std::uint32_t kk = 0; kk < k; ++kk)
            std::memcpy(&pr.b[static_cast<std::size_t>(kk) * np],
                        b_kn + static_cast<std::size_t>(kk) * n + static_cast<std::size_t>(p) * np, np);
        pr.scales.assign(scales + static_cast<std::size_t>(p) * np * groups,
                         scales + static_cast<std::size_t>(p + 1) * np * groups);
    }
    return ps;
}

// Runs every prepared shard, one host thread per shard (threads == parts),
// or serially when threads <= 1.  Returns the number of shards run.
int ref_run(void* handle, int threads) {
    auto* ps = static_cast<std::vector<Problem>*>(handle);
    if (!ps) return 0;
    auto work = [](Problem& pr) { pr.c = ref::cpu_reference(pr.a, pr.b, pr.scales, pr.m, pr.n, pr.k); };
    if (threads <= 1) {
        for (auto& pr : *ps) work(pr);
    } else {
        std::vector<std::thread> pool;
        for (auto& pr : *ps) pool.emplace_back(work, std::ref(pr));
        for (auto& t : pool) t.join();
    }
    return static_cast<int>(ps->size());
}

// Gathers the shard outputs of the last ref_run into c_out [m x n] (double).
void ref_gather(void* handle, double* c_out) {
    auto* ps = static_cast<std::vector<Problem>*>(handle);
    if (!ps || ps->empty()) return;
    const std::uint32_t parts = static_cast<std::uint32_t>(ps->size());
    const std::uint32_t m = (*ps)[0].m, np = (*ps)[0].n, n = np * parts;
    for (std::uint32_t p = 0; p < parts; ++p)
        for (std::uint32_t r = 0; r < m; ++r)
            std::memcpy(c_out + static_cast<std::size_t>(r) * n + static_cast<std::size_t>(p) * np,
                        &(*ps)[p].c[static_cast<std::size_t>(r) * np], np * sizeof(double));
}

void ref_release(void* handle) { delete static_cast<std::vector<Problem>*>(handle); }

}  // extern "C"
