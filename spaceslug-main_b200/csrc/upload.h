// Model-load path of the int4 weights (internal to libspaceslug_b200.so): a
// multi-threaded host packer, and host -> device uploads staged through a
// per-device ring of pinned buffers, with the int4 packing optionally done on
// the device from the logical int8 matrix.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace q4up {

// Reference packing (vulkan-runtime/tests/test_q4gemm.cpp:84-99 layout) of the
// logical matrix w_kn[k*n + col] into packed_out[col*(k/8) + c], on up to
// `threads` host threads (0 = automatic).
void host_pack(const int8_t* w_kn, uint32_t k, uint32_t n, uint32_t* packed_out, int threads = 0);

// Copies `bytes` from host memory to device memory on `stream`.  Pinned
// sources go out as one DMA; pageable sources are copied by several host
// threads into pinned slots while earlier slots are in flight.  The call
// returns once every byte has left the caller's buffer; the device copy
// completes in stream order.
void staged_h2d(int device, void* dst, const void* src, size_t bytes, cudaStream_t stream);

// Packs columns [col_begin, col_begin + ncols) of the logical k x n_total int8
// matrix w_kn (host) into packed_dev (device, ncols * k/8 words, reference
// layout): row blocks of those columns are staged through the pinned slots
// into device scratch and packed there by a kernel.  Returns once the host
// buffer has been read; the packing completes in stream order.
void staged_pack_logical(int device, uint32_t* packed_dev, const int8_t* w_kn, uint32_t k, uint32_t n_total,
                         uint32_t col_begin, uint32_t ncols, cudaStream_t stream);

}  // namespace q4up
