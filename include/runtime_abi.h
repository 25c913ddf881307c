/*
 * Spaceslug native runtime C-ABI, B200 (sm_100a) build.
 *
 * Extends the reference's native/runtime_abi.h (which declares only
 * spaceslug_vector_add) with the int4-dequant GEMM/GEMV + LoRA hot path.  All
 * entry points follow the reference ABI conventions of
 * vulkan-runtime/src/api/lora_delta_api.h:5-13 and sgemm_api.h:5-9:
 *   - extern "C", int return code:
 *       0 ok,
 *       1 invalid arguments (checked before any device work),
 *       2 runtime failure (CUDA error; the reference returns 2 for Vulkan
 *         failures, lora_delta_api.cpp:84),
 *       3 a kernel wait exceeded its time limit (new: the kernels bound every
 *         spin-wait and report instead of hanging);
 *   - plain pointers and sizes, row-major fp32 activations;
 *   - host-pointer entry points are synchronous (they return after the result
 *     is back in host memory), like the reference's;
 *   - no exception ever crosses the ABI.
 * Entry points ending in _device take device pointers and a cudaStream_t
 * passed as void* (NULL = legacy default stream) and are asynchronous.
 *
 * Weight layout ("reference layout", vulkan-runtime/shaders/q4gemm.comp:7-19):
 *   int4 v in [-8, 7] stored as the nibble (v & 0xF); the byte for (k, n) is
 *   pb = n*(K/2) + k/2, even k in the low nibble; bytes are packed 4 per
 *   little-endian uint32 word (K*N/8 words); one fp32 scale per (32-k group,
 *   column) at scales[n*(K/32) + k/32]; w(k, n) = float(v) * scale.
 *
 * Shapes: any M >= 1 and N >= 1; K must be a positive multiple of 32.
 * Device pointers for x, packed and y must be 16-byte aligned.
 *
 * Thread safety: distinct calls may run concurrently from different host
 * threads; one weights handle must not be used by two threads at once.
 */
#ifndef SPACESLUG_RUNTIME_ABI_H
#define SPACESLUG_RUNTIME_ABI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPACESLUG_OK 0
#define SPACESLUG_INVALID_ARGUMENT 1
#define SPACESLUG_RUNTIME_FAILURE 2
#define SPACESLUG_TIMEOUT 3

/* Unchanged from the reference: native/runtime_abi.h:6 / runtime_abi.cpp:3-7
 * (host CPU; returns 1 on a null pointer). */
int spaceslug_vector_add(const float* left, const float* right, float* output, size_t count);

/* Replaces vulkan-runtime/src/api/lora_delta_api.h:8-13 with the same
 * signature, limits and semantics: Y[M,64] = X[M,64] * A[64,R] * B[R,64],
 * fp32 row-major host buffers, 1 <= m <= 128, 1 <= rank <= 8, no alpha/rank
 * scale inside (callers pre-scale B, python/spaceslug/backend.py:666). */
int spaceslug_lora_delta(const float* x, const float* a, const float* b, float* y, uint32_t m, uint32_t rank);

/* Host packer: logical int4 w_kn[k*N + n] in [-8, 7] -> reference layout
 * (K*N/8 words).  Replaces pack_q4 of vulkan-runtime/tests/test_q4gemm.cpp:84-99
 * (and bench/bench_q4gemm.cpp:118-133).  Runs on the host CPU, no GPU needed.
 * Returns 1 for null pointers, k % 32 != 0 or n == 0.  Values outside [-8, 7]
 * are stored as (v & 0xF), exactly like the reference. */
int spaceslug_q4_pack(const int8_t* w_kn, uint32_t k, uint32_t n, uint32_t* packed_out);

/* Device packer (same contract, device pointers, asynchronous on `stream`). */
int spaceslug_q4_pack_device(const int8_t* w_kn, uint32_t k, uint32_t n, uint32_t* packed_out, void* stream);

/* Dequantised weights w_kn[k*N + n] = float(v) * scale in fp32 (one rounding),
 * bit-exact with the reference's dequant (vulkan-runtime/shaders/q4gemm.comp:104-122).
 * Host pointers, synchronous; a debug/check export. */
int spaceslug_q4_dequant(const uint32_t* packed, const float* scales, uint32_t k, uint32_t n, float* w_kn_out);
int spaceslug_q4_dequant_device(const uint32_t* packed, const float* scales, uint32_t k, uint32_t n, float* w_kn_out,
                                void* stream);

/* Y[M x N] = X[M x K] * dequant(W), fp32 in and out, host pointers,
 * synchronous.  The int4 GEMM of vulkan-runtime/shaders/q4gemm.comp (driven by
 * tests/test_q4gemm.cpp:159-425 and bench/bench_q4gemm.cpp:142-396; the
 * reference exports no C symbol for it).  M <= 8 runs the fp32 GEMV, larger M
 * the tcgen05 tensor-core GEMM. */
int spaceslug_q4gemm(const float* x, const uint32_t* packed, const float* scales, float* y, uint32_t m, uint32_t n,
                     uint32_t k);

/* As spaceslug_q4gemm plus the fused LoRA term:
 *   Y = X * dequant(W) + (alpha / rank) * (X * A) * B,
 * A [K x rank], B [rank x N] fp32 row-major (python/spaceslug/lora.py:21-23
 * defines delta = (alpha/rank) * A @ B; the composition replaces
 * python/spaceslug/backend.py:663-667).  1 <= rank <= 64. */
int spaceslug_q4gemm_lora(const float* x, const uint32_t* packed, const float* scales, const float* lora_a,
                          const float* lora_b, uint32_t rank, float alpha, float* y, uint32_t m, uint32_t n,
                          uint32_t k);

/* Device-pointer variant of both of the above (lora_a / lora_b may be NULL
 * with rank 0).  Scratch memory comes from the device's stream-ordered pool. */
int spaceslug_q4gemm_device(const float* x, const uint32_t* packed, const float* scales, const float* lora_a,
                            const float* lora_b, uint32_t rank, float alpha, float* y, uint32_t m, uint32_t n,
                            uint32_t k, void* stream);

/* Device-resident weights (model-load time upload, then many calls), after
 * the persistent-session pattern of vulkan-runtime/src/api/lora_session_api.h:6-14.
 * Pageable host buffers are uploaded through a per-device ring of pinned
 * slots filled by several host threads while earlier slots are in flight;
 * pinned buffers go out as one DMA.
 * The handle keeps columns [col_begin, col_end) of a K x N weight matrix given
 * in the reference layout (host pointers), so a column shard of an N-sharded
 * multi-GPU layer is one contiguous byte range with no repacking.
 * col_begin = 0, col_end = n keeps the whole matrix. */
typedef struct spaceslug_q4_weights spaceslug_q4_weights;
int spaceslug_q4_weights_create(const uint32_t* packed, const float* scales, uint32_t k, uint32_t n,
                                uint32_t col_begin, uint32_t col_end, int device, spaceslug_q4_weights** out);
/* As spaceslug_q4_weights_create, from the logical int4 matrix w_kn[k*n + col]
 * in [-8, 7] (int8 host buffer, the input of pack_q4 in
 * vulkan-runtime/tests/test_q4gemm.cpp:84-99) instead of packed words: row
 * blocks of columns [col_begin, col_end) cross PCIe through pinned staging
 * slots and are packed on the device into the reference layout.  Values
 * outside [-8, 7] are stored as (v & 0xF), like the reference packer. */
int spaceslug_q4_weights_create_logical(const int8_t* w_kn, const float* scales, uint32_t k, uint32_t n,
                                        uint32_t col_begin, uint32_t col_end, int device, spaceslug_q4_weights** out);
/* Copies the handle's packed words ((col_end-col_begin) * k/8, reference
 * layout of those columns) and/or scales ((col_end-col_begin) * k/32) to host
 * buffers; either output may be NULL.  Synchronous. */
int spaceslug_q4_weights_export(const spaceslug_q4_weights* w, uint32_t* packed_out, float* scales_out);
/* Attach (or, with rank 0, detach) a LoRA adapter; lora_b is the full
 * [rank x n] host matrix, the handle keeps its own columns. */
int spaceslug_q4_weights_set_lora(spaceslug_q4_weights* w, const float* lora_a, const float* lora_b, uint32_t rank,
                                  float alpha);
/* Y[m x (col_end-col_begin)] for device pointers, asynchronous on `stream`. */
int spaceslug_q4_weights_run(spaceslug_q4_weights* w, const float* x, float* y, uint32_t m, void* stream);
/* Same with host pointers: copies X in, Y out, synchronous. */
int spaceslug_q4_weights_run_host(spaceslug_q4_weights* w, const float* x, float* y, uint32_t m);
int spaceslug_q4_weights_destroy(spaceslug_q4_weights* w);

/* LoRA training on the handle's adapter, for the fused forward
 *   Y = X * dequant(W) + s * (X * A) * B,  s = alpha / rank, W frozen:
 *   dB = s * (X A)^T dY  [rank x (col_end-col_begin)],  dA = s * X^T (dY B^T)  [k x rank],
 * the reference's lora_gradients (vulkan-runtime/src/api/lora_gradients_api.h:4-6,
 * s = 1 there) for any k, n and rank <= 64.  x [m x k] and dy [m x (col_end -
 * col_begin)] are device pointers; asynchronous on `stream`.  For a column
 * shard, dA is this shard's partial sum: the caller all-reduces it over the
 * shards.  The gradients stay in the handle until the next backward. */
int spaceslug_q4_weights_lora_backward(spaceslug_q4_weights* w, const float* x, const float* dy, uint32_t m,
                                       void* stream);
/* A -= lr * dA, B -= lr * dB (lora_sgd_api.h:4-6), in place on the device. */
int spaceslug_q4_weights_lora_sgd(spaceslug_q4_weights* w, float learning_rate, void* stream);
/* AdamW with decoupled weight decay and bias-corrected moments (kept in the
 * handle; set_lora resets them):  m = b1 m + (1-b1) g,  v = b2 v + (1-b2) g^2,
 * p -= lr * ((m / (1-b1^t)) / (sqrt(v / (1-b2^t)) + eps) + wd * p). */
int spaceslug_q4_weights_lora_adamw(spaceslug_q4_weights* w, float learning_rate, float beta1, float beta2, float eps,
                                    float weight_decay, void* stream);
/* Host copies of the adapter and its last gradients (any output may be NULL);
 * synchronises the device. */
int spaceslug_q4_weights_get_lora(const spaceslug_q4_weights* w, float* a_out, float* b_out, float* da_out,
                                  float* db_out);

/* The reference's hidden-64 training ABI, same contracts and return codes:
 * dA = X^T dY B^T and dB = (X A)^T dY for X/dY [m x 64], A [64 x rank],
 * B [rank x 64], 1 <= m <= 128, 1 <= rank <= 8 (lora_gradients_api.h:4-6);
 * A -= lr dA, B -= lr dB (lora_sgd_api.h:4-6); and one training step: delta
 * forward into y, gradients at the old A/B, SGD (lora_train_api.h:4-10).
 * Host pointers, synchronous. */
int spaceslug_lora_gradients(const float* x, const float* dy, const float* a, const float* b, float* da, float* db,
                             uint32_t m, uint32_t rank);
int spaceslug_lora_sgd(float* a, float* b, const float* da, const float* db, float learning_rate, uint32_t rank);
int spaceslug_lora_train_step(const float* x, const float* dy, float* a, float* b, float* y, float learning_rate,
                              uint32_t m, uint32_t rank);

/* No counterpart in the reference.  The decode GEMV with the fused LoRA term
 * (device pointers, asynchronous on `stream`, same result as
 * spaceslug_q4gemm_device with the same arguments) for callers that cannot
 * allocate device memory: serving loops that forbid allocation on the hot
 * path (an allocation can stall or synchronise the device), plugin hosts that
 * keep all device memory for themselves.  It allocates nothing: its
 * only scratch, T = X*A, lives in a fixed 2 KB static device array, so
 * 1 <= m <= 8 and 1 <= rank <= 64; and, as for the decode GEMV itself, K/32
 * must split into 1, 2, 4 or 8 equal slices of at most 32 scale groups (every
 * K <= 1024 and every multiple of 256 up to 8192 does); other shapes return 1.  The first call on each device
 * sets up the array's address (make it before any stream capture).  All calls
 * on a device share the array: calls that overlap on the GPU race.  The call
 * returns before the kernels run, so a kernel wait that runs out of time is
 * reported by spaceslug_q4_device_status(device), which allocates nothing. */
int spaceslug_q4gemv_lora_noalloc(const float* x, const uint32_t* packed, const float* scales, const float* lora_a,
                                  const float* lora_b, uint32_t rank, float alpha, float* y, uint32_t m, uint32_t n,
                                  uint32_t k, void* stream);

/* Operand type of the tensor-core path: 0 = f16 with exact power-of-two
 * row/column exponents (default), 1 = bf16.  Returns the previous value, or
 * -1 for an invalid type. */
int spaceslug_q4_set_operand_type(int type);

/* Tensor-core GEMM kernel selection for M > 8: 0 = automatic (default),
 * 1 = single-CTA kernel with 128-row tiles, 2 = CTA-pair (cta_group::2)
 * kernel, 3 = single-CTA kernel with 256-row tiles.  Results are the
 * same up to fp32 summation order.  Returns the previous value, or -1 for an
 * invalid value. */
int spaceslug_q4_set_gemm_variant(int variant);

/* Decode (M <= 8) kernel selection: 0 = automatic (default: the whole-tile
 * GEMV where the shape allows it, else the streamed ring), 1 = CUDA-core GEMV
 * with a streamed shared-memory ring, 2 = tcgen05 tensor-core decode,
 * 3 = CUDA-core GEMV with the whole tile resident, 4 = integer-tensor-core
 * (mma.sync s8) GEMV with exact int8 limbs of X (K % 1024 == 0).  A variant the shape does not allow falls
 * back to the automatic choice.  Results agree to fp32 summation order.
 * Returns the previous value, or -1 for an invalid value. */
int spaceslug_q4_set_decode_variant(int variant);

/* Reads and clears the kernel status words of `device` (0 = no kernel wait
 * has timed out since the last call): the word of the regular entry points
 * and the one of spaceslug_q4gemv_lora_noalloc.  Synchronises the device.
 * Allocates nothing (a device no regular entry point has run on has no
 * word of its own yet and reads as 0), so the asynchronous entry points,
 * the no-allocation one included, report a timeout through this call. */
int spaceslug_q4_device_status(int device);

/* Test hook (no reference counterpart), current device: sets the time limit
 * of the decode kernels' bounded waits to wait_limit_ns (0 = the default 2 s)
 * and, with stall != 0, makes one warp in every CTA of those kernels wait on
 * a barrier phase that nothing arms, so that the wait runs out, the kernel
 * records the timeout and returns, and the call reports code 3 (synchronous
 * entry points) or spaceslug_q4_device_status reports it (asynchronous ones).
 * Synchronises the device first.  For tests of the timeout path only. */
int spaceslug_q4_debug_wait_test(uint64_t wait_limit_ns, int stall);

/* Number of kernels this library has launched since load (all devices). */
uint64_t spaceslug_q4_launch_count(void);

/* Human-readable description of the last non-zero return code on this thread. */
const char* spaceslug_last_error(void);

/* fp32 row-major C[m x n] = A[m x k] * B[k x n], host pointers, synchronous:
 * the reference's spaceslug_sgemm (vulkan-runtime/src/api/sgemm_api.h:5-9), same
 * checks (M, N % 64 == 0, K % 32 == 0) and codes; *max_relative_error is set
 * to 0 as the reference does.  Computed on the tcgen05 tensor cores with
 * fp32-level accuracy: each operand split into TF32 hi + lo parts, three TF32
 * MMAs per product (hi*hi + hi*lo + lo*hi) accumulated in fp32. */
int spaceslug_sgemm(const float* a, const float* b, float* c, uint32_t m, uint32_t n, uint32_t k,
                    float* max_relative_error);
/* Same product for device pointers, any positive m, n, k, asynchronous on
 * `stream`; the TF32 hi/lo planes of the operands take stream-ordered scratch. */
int spaceslug_sgemm_device(const float* a, const float* b, float* c, uint32_t m, uint32_t n, uint32_t k, void* stream);

/* spaceslug_q4_weights_run with a row pitch: Y[i][j] at y[i * ld_y + j] for
 * j < the handle's column count; other columns of the pitched rows are not
 * written (a rank's column shard straight into the full row-major Y).  x
 * 16-byte aligned, y 4-byte aligned, ld_y >= the handle's column count. */
int spaceslug_q4_weights_run_strided(spaceslug_q4_weights* w, const float* x, float* y, uint32_t m, uint64_t ld_y,
                                     void* stream);

/* spaceslug_q4_weights_run_strided that also stores the same rows and columns
 * of Y into each of npeers (<= 7) other GPUs' buffers, peer_y[q] pointing at
 * the place that corresponds to y (host array of device pointers mapped with
 * spaceslug_ipc_open; same row pitch).  No reference counterpart: the
 * N-sharded all-gather of Y fused into the GEMM.  The pair kernel pushes each
 * finished 32 x 32 block from its epilogue while the next tile computes
 * (16-byte aligned y and peers, K % 128 == 0, N % 4 == 0); other shapes run
 * the GEMM, then push the whole block.  The caller orders the peers' use of
 * their buffers around the call (for instance with a collective before and
 * after it). */
int spaceslug_q4_weights_run_push(spaceslug_q4_weights* w, const float* x, float* y, uint32_t m, uint64_t ld_y,
                                  float* const* peer_y, uint32_t npeers, void* stream);
/* Caps the SMs a GEMM launch of this handle occupies (0: all, else >= 2), so
 * that kernels on other streams (an exchange running beside the GEMM) find
 * free SMs.  Decode-sized launches (m <= 8) ignore it. */
int spaceslug_q4_weights_set_sm_budget(spaceslug_q4_weights* w, uint32_t sms);
/* Stores rows [0, rows) x columns [0, width) of the pitched fp32 block at
 * `src` (row pitch ld floats) to the same offsets in npeers (<= 7) peer-mapped
 * buffers (peer_dst: host array of device pointers), with `ctas` CTAs of plain
 * global stores over NVLink; asynchronous on `stream`. */
int spaceslug_push_rows(const float* src, float* const* peer_dst, uint32_t npeers, uint32_t rows, uint32_t width,
                        uint64_t ld, uint32_t ctas, void* stream);

/* CUDA IPC between the ranks of one node (no reference counterpart).
 * export: 64-byte handle of the device allocation holding `ptr` and the byte
 * offset of ptr inside it.  open: maps a peer's allocation on `device`
 * (peer access enabled on first use); *ptr = mapped base + offset, *base is
 * what close takes. */
int spaceslug_ipc_export(const void* ptr, void* handle64, uint64_t* offset);
int spaceslug_ipc_open(const void* handle64, uint64_t offset, int device, void** ptr, void** base);
int spaceslug_ipc_close(void* base);
/* Pitched copy of `rows` rows of width_bytes between any two device (or
 * peer-mapped) addresses, asynchronous on `stream` (a copy engine, no SMs). */
int spaceslug_copy_2d(void* dst, uint64_t dpitch, const void* src, uint64_t spitch, uint64_t width_bytes,
                      uint64_t rows, void* stream);

/* N-sharded GEMM exchange (no reference counterpart: the reference runs on one
 * device).  After an all-gather of equal-width column shards of Y, the
 * gathered buffer is rank-major [parts][rows][width]; this writes it into
 * rows [rows][ld_y] of row-major Y, columns [0, n_total) (n_total <=
 * parts * width; the last shard's padding columns are dropped).  Device
 * pointers, asynchronous on `stream`. */
int spaceslug_shards_relayout(const float* gathered, float* y, uint32_t parts, uint32_t rows, uint32_t width,
                              uint32_t n_total, uint64_t ld_y, void* stream);

/* ---- CQ4 (Cactus-Quants) ------------------------------------------------
 * C[M x N] = A'[M x K] * W'^T in fp16 storage with fp32 accumulation, where
 * A' is the activation transformed into the code basis and
 * W'[n][k] = norm(n, k / group_size) * codebook[idx(n, k)]: the reference's
 * cactus_quant_matmul (vulkan-runtime/src/cactus/cactus_x86.cpp:384-397),
 * which its GPU path runs as transform_act -> dequant_w -> sgemm_f16_am
 * (bench/bench_cq4gemm.cpp).  The matrix description is field for field the
 * reference's CactusQuantMatrixBridge (src/cactus/cactus_x86_bridge.h), so a
 * pointer to one can be passed as is; fp16 values are IEEE binary16 bits.
 * Supported: bits == 4; K % 32 == 0; Hadamard mode with a power-of-two
 * group_size in [32, 256] and K == group_size * num_groups, or the
 * orthogonal mode (one group spanning K, dense rotation [K][K]);
 * INTERLEAVED_4ROW panels need N % 4 == 0.  The product runs on the tcgen05
 * GEMM with the codebook applied while the weights are dequantised. */
#define SPACESLUG_CQ4_FLAG_ORTHOGONAL 4u       /* CACTUS_BRIDGE_QUANT_FLAG_ORTHOGONAL */
#define SPACESLUG_CQ4_FLAG_INTERLEAVED_4ROW 8u /* CACTUS_BRIDGE_QUANT_FLAG_INTERLEAVED_4ROW */
typedef struct spaceslug_cq4_matrix {
    uint32_t bits;
    uint32_t k;
    uint32_t n;
    uint32_t group_size;
    uint32_t num_groups;
    uint32_t flags;
    const uint16_t* codebook;          /* [2^bits] fp16 */
    const uint16_t* input_scale;       /* [K] fp16 or NULL */
    const uint16_t* input_scale_recip; /* [K] fp16 or NULL (takes precedence) */
    const uint16_t* norms;             /* [N * num_groups] fp16, stored layout (panel-major when interleaved) */
    const uint8_t* packed_indices;     /* LSB-first 4-bit indices, or 4-row interleaved panels */
    const int8_t* left_signs;          /* [group_size] +-1 or NULL */
    const int8_t* right_signs;         /* [group_size] +-1 or NULL */
    const uint32_t* permutation;       /* [group_size] or NULL */
    const uint16_t* rotation;          /* [K * K] fp16, orthogonal mode only */
    const int8_t* expanded;            /* unused */
    const float* norm_f32;             /* unused */
} spaceslug_cq4_matrix;
typedef struct spaceslug_cq4_weights spaceslug_cq4_weights;
/* Uploads a CQ4 matrix (host pointers) to `device`. */
int spaceslug_cq4_weights_create(const spaceslug_cq4_matrix* m, int device, spaceslug_cq4_weights** out);
/* C = cactus_quant_matmul(W, A): a [m x K] and c [m x N] fp16 device
 * pointers, asynchronous on `stream`. */
int spaceslug_cq4_matmul(spaceslug_cq4_weights* w, const uint16_t* a, uint16_t* c, uint32_t m, void* stream);
/* Same with host pointers, synchronous. */
int spaceslug_cq4_matmul_host(spaceslug_cq4_weights* w, const uint16_t* a, uint16_t* c, uint32_t m);
/* The code-basis activations alone (fp16, [m x K]), host pointers: the
 * reference's transform_act output (shaders/transform_act.comp). */
int spaceslug_cq4_transform_host(spaceslug_cq4_weights* w, const uint16_t* a, uint16_t* a_out, uint32_t m);
int spaceslug_cq4_weights_destroy(spaceslug_cq4_weights* w);

#ifdef __cplusplus
}
#endif

#endif /* SPACESLUG_RUNTIME_ABI_H */
