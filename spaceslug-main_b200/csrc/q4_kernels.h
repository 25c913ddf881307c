// Launch interfaces of the sm_100a kernels (internal to libspaceslug_b200.so;
// the public C-ABI is include/runtime_abi.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace q4 {

// 16-bit operand type of the tensor-core (prefill) path.
enum class Operand16 : int { kF16 = 0, kBF16 = 1 };

struct GemvArgs {
    CUtensorMap tmap_w;      // packed weights as uint32 [N][K/8], box (K/S/8) x 16 columns, no swizzle
    const float* x;          // [M][K] fp32, device
    const float* scales;     // [N][K/32], device
    float* y;                // [M][N] fp32, device
    int M, N, K;
    int cluster_k;           // CTAs per cluster = number of K slices
    int clusters;            // grid = cluster_k * clusters CTAs
    int cols_per_cluster;
    const float* lora_t;     // [M][rank] = X*A (fp32) or nullptr
    const float* lora_b;     // [rank][N] or nullptr
    int rank;
    float lora_scale;        // alpha / rank
    int* status;             // kernel status word (0 = ok)
};
int launch_gemv(const GemvArgs& a, cudaStream_t stream);
// Test hooks of the decode kernels, for the current device: the wait limit of
// every bounded wait of that kernel file (ns) and, with stall != 0, one warp
// per CTA that waits on a barrier phase nothing arms (the wait runs out).
int gemv_ring_set_wait_test(unsigned long long limit_ns, int stall);
int gemv_tile_set_wait_test(unsigned long long limit_ns, int stall);
int gemv_imma_set_wait_test(unsigned long long limit_ns, int stall);
// Integer-tensor-core GEMV (M <= 8, K % 1024 == 0): 16-column tiles, K split
// over a cluster of cluster_k CTAs, tiles_per_cta tiles and kparts warps per
// tile in each CTA.  16-byte aligned x, packed and scales.
struct GemvImmaArgs {
    CUtensorMap tmap_w;      // packed uint32 [N][K/8], box 32 words x (16 tiles_per_cta), 128B swizzle
    CUtensorMap tmap_s;      // scales fp32 [N][K/32], box 32 x (16 tiles_per_cta), 128B swizzle
    CUtensorMap tmap_x;      // X fp32 [M][K], box 256 x M, no swizzle
    float* y;                // [M][N]
    int M, N, K;
    int cluster_k;           // S
    int clusters;            // cluster c holds tiles [c*tiles_total/clusters, (c+1)*tiles_total/clusters)
    int tiles_total;         // ceil(N / 16)
    int tiles_per_cta;       // T = ceil(tiles_total / clusters)
    int kparts;              // P
    const float* lora_t;     // [M][rank] or nullptr
    const float* lora_b;     // [rank][N] or nullptr
    int rank;
    float lora_scale;
    int* status;
};
bool gemv_imma_geometry(int sm_count, int M, int N, int K, int* S, int* clusters, int* T, int* P);
size_t gemv_imma_smem_bytes(int M, int K, int S, int T, int P);
int launch_gemv_imma(const GemvImmaArgs& a, cudaStream_t stream);
// Tensor-core decode (M <= 8): col_blocks blocks of <= 128 columns, each a
// cluster of cluster_k CTAs splitting K into slices of <= 1024.
struct DecodeArgs {
    CUtensorMap tmap_w;      // packed uint32 [N][K/8], box 32 words x box_rows, 128B swizzle
    CUtensorMap tmap_x;      // X fp32 viewed as [M*K/256][256], box 256 x (K/cluster_k/256)
    const float* scales;     // [N][K/32], 16-byte aligned
    float* y;                // [M][N]
    int M, N, K;
    int cluster_k;           // = decode_split(M, K)
    int col_blocks;          // G: block g holds columns [g*N/G, (g+1)*N/G)
    int box_rows;            // multiple of 8, >= ceil(N/G), <= 128
    const float* lora_t;     // [M][rank] or nullptr
    const float* lora_b;     // [rank][N] or nullptr
    int rank;
    float lora_scale;
    int* status;
};
int decode_split(int M, int K);  // cluster size, 0 = shape not supported
size_t decode_smem_bytes(int M, int K, int S, int box_rows);
int decode_max_clusters(int M, int K, int S, int box_rows);  // co-resident clusters (one wave)
int decode_rows();
int decode_x_box();
int launch_decode(const DecodeArgs& a, cudaStream_t stream);
// Whole-tile GEMV (M <= 8): col_blocks blocks of <= 32 columns x K/S per CTA,
// every load issued at entry.  Needs K % (256 * S) == 0 and 16-byte aligned x,
// packed and scales.
struct GemvTileArgs {
    CUtensorMap tmap_w;      // packed uint32 [N][K/8], box 32 words x box_rows, 128B swizzle
    CUtensorMap tmap_s;      // scales fp32 [N][K/32], box 32 x box_rows, 128B swizzle
    CUtensorMap tmap_x;      // X fp32 viewed as [M*K/256][256], box 256 x (K/S/256)
    float* y;                // [M][N]
    int M, N, K;
    int cluster_k;           // S: CTAs per cluster splitting K
    int col_blocks;          // G: block g holds columns [g*N/G, (g+1)*N/G)
    const float* lora_t;     // [M][rank] or nullptr
    const float* lora_b;     // [rank][N] or nullptr
    int rank;
    float lora_scale;
    int* status;
};
bool gemv_tile_supported(int M, int K, int S);
size_t gemv_tile_smem_bytes(int M, int K, int S);
// Column blocks for N on sm_count SMs, and the rows of its boxes (<= 32).
int gemv_tile_col_blocks(int N, int sm_count);
int gemv_tile_box_rows(int N, int col_blocks);
int gemv_tile_box_k();
int gemv_tile_scale_box_groups();
int launch_gemv_tile(const GemvTileArgs& a, cudaStream_t stream);
size_t gemv_smem_bytes(int M, int K, int cluster_k, int cols_per_cluster);
int gemv_chunk_columns();
// Max co-resident clusters of the GEMV for these parameters (0 on error).
int gemv_max_active_clusters(int M, int K, int cluster_k, int cols_per_cluster);

// Device pointers of up to kMaxPeers other GPUs' buffers (peer mappings).
constexpr int kMaxPeers = 7;
struct PeerPtrs {
    float* p[kMaxPeers];
};

struct GemmArgs {
    CUtensorMap tmap_x16;     // [M][K] 16-bit, box 64 x (128 * halves), 128B swizzle
    CUtensorMap tmap_w;       // packed as uint32 [N][K/8]: box 8 x 128 unswizzled (single-CTA), 16 x 128 64B-swizzled (pair)
    CUtensorMap tmap_s;       // pair kernel: scales fp32 [N][K/32], box 4 x 128 (needs K % 128 == 0)
    CUtensorMap tmap_y;       // pair kernel: Y fp32 [M][N], box 32 x 32 (needs N % 4 == 0, 16-byte aligned Y)
    CUtensorMap tmap_t;       // LoRA-stage A operand, bf16 [M][64*stages], box 64 x (128 * halves), 128B swizzle
    const float* scales;      // [N][K/32]
    const int* col_exp;       // [N] power-of-two exponent applied to the column's scales, or nullptr
    const int* row_exp;       // [M] power-of-two exponent applied to X rows, or nullptr
    float* y;                 // [M][N]
    int M, N, K;
    Operand16 op;
    int halves;               // output tile rows = 128 * halves (1 or 2); tile columns = 128
    int sm_count;             // persistent grid size limit
    const float* lora_t;      // [M][rank] fp32 or nullptr
    const float* lora_b;      // [rank][N] fp32
    int rank;
    float lora_scale;
    int lora_stages;          // single-CTA kernel: ceil(rank/16) bf16 k-stages (0 = no LoRA); the pair kernel
                              // adds the LoRA term in its epilogue from lora_t
    const uint32_t* lut = nullptr;  // single-CTA kernel, f16 only: CQ4 codebook pairs (256 words); the
                                    // scales are then the norms and W = RN16(codebook[idx] * norm)
    void* y16 = nullptr;            // single-CTA kernel: fp16 [M][N] output instead of y
    int ksplit = 1;           // pair kernel: 1, or 2 = each tile as two K halves reduce-added into a zeroed Y
    PeerPtrs peers{};         // pair kernel, ksplit 1: every Y block also stored to these peers' Y ...
    int npeers = 0;
    long long peer_ld = 0;    // ... at the same offsets, row pitch peer_ld floats (= Y's)
    int* status;              // kernel status word (0 = ok)
};
int launch_gemm(const GemmArgs& a, cudaStream_t stream);
int gemm_tiles(int M, int N, int halves);
// CTA-pair (cta_group::2) variant, 256 x 256 tiles; X tensor map box 64 x 128.
int launch_gemm_pair(const GemmArgs& a, int max_pairs, cudaStream_t stream);
int gemm_pair_tiles(int M, int N);
int gemm_pair_max_active(Operand16 op);

// fp32 -> 16-bit cast of X with per-row power-of-two exponents (row_exp may be
// nullptr: plain round-to-nearest cast).
int launch_cast_x(const float* x, void* x16, int* row_exp, int M, int K, Operand16 op, cudaStream_t stream);
// Per-column exponent f_n so that 8 * max_g |scale[n][g]| * 2^f_n lies in [2^13, 2^14).
int launch_col_exp(const float* scales, int* col_exp, int N, int K, cudaStream_t stream);
// Bit-exact dequant w[k*N + n] = float(v) * scale (fp32).
int launch_dequant(const uint32_t* packed, const float* scales, float* w_kn, int K, int N, cudaStream_t stream);
// Device packer: logical int8 b[k*N + n] in [-8,7] -> reference layout.
int launch_pack(const int8_t* b_kn, uint32_t* packed, int K, int N, cudaStream_t stream);
// T[M][rank] = X[M][K] * A[K][rank] in fp32.  With `partial` (scratch of
// lora_xa_chunks(K) * M * rank floats) K is split over CTAs and reduced in a
// second kernel in fixed order; with nullptr one pass per (32 rows, 16 ranks).
// With `partial` and t_op_bits != nullptr, the reduction also writes the GEMM's
// LoRA-stage operand: bf16 [M][64 * ceil(rank/16)], per 16 ranks a block
// [hi | lo | hi | 0] of T[m][:] * 2^row_exp[m] (row_exp may be nullptr).
int launch_lora_xa(const float* x, const float* a, float* t, int M, int K, int rank, cudaStream_t stream,
                   float* partial = nullptr, const int* row_exp = nullptr, uint16_t* t_op_bits = nullptr);
int lora_xa_chunks(int K);
// Y[m][n] (row pitch ld) += s * T[m][:] . B[:][n] (B [rank][N], rank <= 64):
// the LoRA term of a split-K GEMM that left it out of its epilogue.
int launch_lora_add(const float* t, const float* b, float* y, int M, int N, long long ld, int rank, float s,
                    cudaStream_t stream);
// All-gathered column shards [parts][rows][width] (rank-major) -> rows
// [rows][ld_y] of row-major Y, columns [0, n_total) (the last shard may be
// partly padding).  HBM-bound copy; float4 when every address is aligned.
// Push of a pitched fp32 row block to the same offset in peers' buffers
// (peer-mapped device pointers) by `ctas` CTAs of plain global stores.
int launch_push_rows(const float* src, const PeerPtrs& peers, int npeers, int rows, int width, long long ld, int ctas,
                     cudaStream_t stream);
// n floats src -> dst by a small kernel (either side device memory or mapped
// pinned host memory), plus the status word when status_src is given.  With
// done_flag (mapped host word) and done_count (device counter, 0 between
// launches), the last CTA sets *done_flag = 1 once every store is visible to
// the host.
int launch_copy_words(const float* src, float* dst, long long n, const int* status_src, int* status_dst,
                      cudaStream_t stream, int* done_flag = nullptr, unsigned* done_count = nullptr);
int launch_shards_relayout(const float* gathered, float* y, int parts, int rows, int width, int n_total,
                           long long ld_y, cudaStream_t stream);
// CQ4 activation transform into the code basis, fp16 [M][K] -> fp16 [M][K]:
// Hadamard groups of gs in {32, 64, 128, 256} (rotation == nullptr) or the
// dense orthogonal rotation [K][K] fp16.  lsign / rsign ([gs], +-1) and perm
// ([gs]) may be nullptr.
int launch_cq4_transform(const void* a, void* a_out, const float* recip, const float* lsign, const float* rsign,
                         const uint32_t* perm, const void* rotation, int M, int K, int gs, float inv_sqrt,
                         cudaStream_t stream);
int launch_f32_to_f16(const float* y, void* c, long long count, cudaStream_t stream);
// CQ4 decode (1 <= M <= 8, M * K * 2 <= 192 KB): C fp16 [M][N] from the
// indices [N][K/8 words], the expanded norms [N][K/32] and the codebook cbf
// [16] (fp32).  fused_gs = 0: `a` holds the transformed activations A';
// fused_gs = group size (32..256): `a` holds the raw activations and every
// CTA applies the Hadamard transform itself.
struct Cq4GemvArgs {
    const void* a;
    const uint32_t* packed;
    const float* scales;
    const float* cbf;
    const float* recip;
    const float* lsign;
    const float* rsign;
    const uint32_t* perm;
    float inv_sqrt;
    int fused_gs;
    void* c;
    int M, N, K;
};
int launch_cq4_gemv(const Cq4GemvArgs& g, cudaStream_t stream);
// LoRA training (lora_train.cu): dB = s T^T dY, dA = s X^T (dY B^T) with
// T = X A, for X [M][K], dY [M][N], A [K][r], B [r][N] (device, fp32).
struct LoraBackwardArgs {
    const float* x;
    const float* dy;
    const float* lora_a;
    const float* lora_b;
    float* da;       // [K][r]
    float* db;       // [r][N]
    float* scratch;  // lora_backward_scratch_floats(M, K, N, r) floats
    int M, K, N, rank;
    float scale;
};
size_t lora_backward_scratch_floats(int M, int K, int N, int rank);
int launch_lora_backward(const LoraBackwardArgs& a, cudaStream_t stream);
// LoRA gradients on the tcgen05 tensor cores (lora_tc.cu).  A problem is
// partial[split][row][rp] of D[R x r] = sum over l < L of Aop[row][l] Bop[j][l];
// tm_a: Aop fp32 with 128B swizzle, rows of D = source rows (mn_major = 0:
// dims {L, R}, box 32 x 128) or rows of D contiguous in the source
// (mn_major = 1: dims {R, L}, box 32 x 32); tm_b: the stacked TF32 hi / lo
// planes of Bop, dims {L, 2 rp}, box 32 x 2 rp.  One launch walks the work
// units of one or two problems of the same form.
struct LoraTcProblem {
    CUtensorMap tm_a, tm_b;
    float* partial;  // [splits][R][rp]
    int R, L, splits;
};
struct LoraTcPass {
    LoraTcProblem prob[2];
    int count;  // 1 or 2
    int mn_major, rp, sm_count;
    int* status;
};
int lora_tc_rp(int rank);  // padded rank: 8, 16, 32 or 64
// l ranges per 128-row tile for `count` problems sharing one launch
void lora_tc_plan(int count, const int* R, const int* L, int sm_count, int* splits);
int launch_lora_tc_pass(const LoraTcPass& p, cudaStream_t stream);
// v[row][j] = sum of the splits in order; mode 0: stacked TF32 planes of the
// transpose ([2 rp][ld]); mode 1: s * transpose ([r][ld]); mode 2: s * rows
// ([R][ld]); mode 3: stacked planes of a row-major [r][R] source (pitch =
// its row pitch, splits = 1).
struct LoraTcFinalize {
    const float* src;
    int splits, R, pitch, r, mode;
    float s;
    float* out;
    long long ld;
};
int launch_lora_tc_finalize(const LoraTcFinalize* f, int count, int rp, cudaStream_t stream);
int launch_sgd(float* p, const float* g, float lr, long long count, cudaStream_t stream);
int launch_adamw(float* p, const float* g, float* m1, float* m2, float lr, float beta1, float beta2, float eps,
                 float wd, int step, long long count, cudaStream_t stream);
// fp32 GEMM on tcgen05 with 3xTF32 (sgemm_tc.cu).  The operands are first
// split into TF32 hi / lo planes in K-major layout ([out_rows][ld] fp32, K
// contiguous): launch_split_planes writes the planes of a row-major
// [rows][cols] matrix (transpose = false: plane row i = source row i) or of
// its transpose (transpose = true: plane row i = source column i); rows and
// columns past the source's, up to out_rows and ld, are zero.
int launch_split_planes(const float* src, int rows, int cols, long long ld_src, bool transpose, float* hi, float* lo,
                        int out_rows, long long ld_out, cudaStream_t stream);
struct SgemmTcArgs {
    CUtensorMap tm_ahi, tm_alo;  // A planes [M rounded up to 128][ld] fp32 (ld % 32 == 0), box 32 x 128, 128B swizzle
    CUtensorMap tm_bhi, tm_blo;  // B^T planes [N rounded up to bn][ld] fp32, box 32 x bn, 128B swizzle
    float* c;                    // C[M][N], row pitch ldc floats: C = alpha * A B
    int M, N, K;
    long long ldc;
    float alpha;
    int bn;                      // tile columns: sgemm_tc_bn(N)
    int* status;
};
int sgemm_tc_bn(int N);
int launch_sgemm_tc(const SgemmTcArgs& a, cudaStream_t stream);
// The CTA-pair form for large problems: 256 x 256 tiles of C, the A and B^T
// planes padded to whole 256-row tiles and mapped with 32 x 128 boxes (each
// CTA loads 128 rows); at most max_pairs co-resident pairs (persistent).
int sgemm_pair_tiles(int M, int N);
int sgemm_pair_max_active();
int launch_sgemm_pair(const SgemmTcArgs& a, int max_pairs, cudaStream_t stream);
// Legacy spaceslug_lora_delta: Y[M,64] = X[M,64] A[64,R] B[R,64].
int launch_lora_delta64(const float* x, const float* a, const float* b, float* y, int M, int rank,
                        cudaStream_t stream);

}  // namespace q4
