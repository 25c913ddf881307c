// C-ABI wrapper around the reference's own CQ4 CPU oracle (cactus_quant_matmul
// and its Hadamard activation transform).
//
// TEST INFRASTRUCTURE ONLY (the shipped library never loads it).  The
// reference code is NOT in this repository: this file includes
// vulkan-runtime/src/cactus/cactus_x86.cpp from the read-only reference
// checkout (oracle/Makefile passes -I .../vulkan-runtime/src) and compiles it
// unmodified with g++.  That file stores fp16 as clang's __fp16 and refuses
// other compilers (cactus_x86.h:25-27); its own header comment names the
// gcc route: _Float16 has the same storage and the same round-to-nearest-even
// conversions.  So, after every standard header the reference uses has been
// included normally, __fp16 is mapped to _Float16 and the clang check is
// satisfied for the reference's own translation unit only.
#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <limits>
#include <random>
#include <vector>

#define __clang__ 1
#define __fp16 _Float16
#include "cactus/cactus_x86.cpp"
#undef __fp16
#undef __clang__

namespace {
CactusQuantMatrix make_matrix(uint32_t bits, uint32_t k, uint32_t n, uint32_t gs, uint32_t ng, uint32_t flags,
                              const uint16_t* codebook, const uint16_t* input_scale,
                              const uint16_t* input_scale_recip, const uint16_t* norms, const uint8_t* packed,
                              const int8_t* left, const int8_t* right, const uint32_t* perm,
                              const uint16_t* rotation) {
    auto h = [](const uint16_t* p) { return reinterpret_cast<const _Float16*>(p); };
    CactusQuantMatrix w{};
    w.bits = bits;
    w.K = k;
    w.N = n;
    w.group_size = gs;
    w.num_groups = ng;
    w.flags = flags;
    w.codebook = h(codebook);
    w.input_scale = h(input_scale);
    w.input_scale_recip = h(input_scale_recip);
    w.norms = h(norms);
    w.packed_indices = packed;
    w.left_signs = left;
    w.right_signs = right;
    w.permutation = perm;
    w.rotation = h(rotation);
    w.expanded = nullptr;
    w.norm_f32 = nullptr;
    return w;
}
}  // namespace

extern "C" {

// C[M x N] (fp16 bits) = cactus_quant_matmul(W, A[M x K] fp16 bits).
void ref_cq4_quant_matmul(uint32_t bits, uint32_t k, uint32_t n, uint32_t gs, uint32_t ng, uint32_t flags,
                          const uint16_t* codebook, const uint16_t* input_scale, const uint16_t* input_scale_recip,
                          const uint16_t* norms, const uint8_t* packed, const int8_t* left, const int8_t* right,
                          const uint32_t* perm, const uint16_t* rotation, const uint16_t* a, uint32_t m,
                          uint16_t* c) {
    const CactusQuantMatrix w = make_matrix(bits, k, n, gs, ng, flags, codebook, input_scale, input_scale_recip,
                                            norms, packed, left, right, perm, rotation);
    cactus_quant_matmul(&w, reinterpret_cast<const _Float16*>(a), m, reinterpret_cast<_Float16*>(c));
}

// Code-basis activations (fp32) of one row, group by group, through the
// reference's transform_hadamard_group.
void ref_cq4_transform_hadamard_row(uint32_t k, uint32_t gs, uint32_t ng, const uint16_t* input_scale,
                                    const uint16_t* input_scale_recip, const int8_t* left, const int8_t* right,
                                    const uint32_t* perm, const uint16_t* a_row, float* basis_out) {
    const CactusQuantMatrix w = make_matrix(4, k, 1, gs, ng, 0, nullptr, input_scale, input_scale_recip, nullptr,
                                            nullptr, left, right, perm, nullptr);
    for (uint32_t g = 0; g < ng; ++g)
        vulkan_runtime::cactus_x86::transform_hadamard_group(w, reinterpret_cast<const _Float16*>(a_row) + g * gs, g,
                                                             basis_out + g * gs);
}

}  // extern "C"
