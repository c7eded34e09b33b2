// Internal host-side interface between the C-ABI layer (capi.cu) and the kernel
// translation units.  Not installed; the public interface is include/metallora_b200.h.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

namespace mlora {

// Element type of the 16-bit tensor-core operands.
enum class Elt { kBF16 = 0, kF16 = 1 };

// Thread-local detail of the last failure (read by mlora_last_error_message).
void set_error(const std::string& msg);

// Encodes a 2-D row-major tensor map over a 16-bit tensor [outer, inner] with
// row stride `row_stride_elems` and a (box_inner x box_outer) box, 128-byte
// swizzle, zero fill out of bounds.  Returns false (with set_error) on failure.
bool make_tmap_2d_16b(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer);
// General 2-D tensor map (element type/size given; 128-byte swizzle or none).
bool make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, uint32_t esize, const void* base,
                  uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                  uint32_t box_outer, bool swizzle128);

// ---- launch accounting / opt-in profiling ----------------------------------
// Kernel kinds for mlora_profile_* (index into the per-kind totals).
enum KernelKind : int {
  kKindGemm = 0,
  kKindRank = 1,
  kKindWgrad = 2,
  kKindElementwise = 3,
  kKindQuant = 4,
  kKindGemv = 5,
  kKindOptim = 6,
  kNumKinds = 7,
};
// Records one launch of `kind` on `stream`: bumps the launch counter and, while
// profiling is enabled, brackets the launch with CUDA events.  Construct right
// before the launch; the destructor records the stop event.
class LaunchScope {
 public:
  LaunchScope(int kind, cudaStream_t stream);
  ~LaunchScope();
  LaunchScope(const LaunchScope&) = delete;
  LaunchScope& operator=(const LaunchScope&) = delete;

 private:
  int kind_;
  cudaStream_t stream_;
  cudaEvent_t stop_ = nullptr;
};

// Device status word of the current device (kernels record bounded-wait
// timeouts here).
uint32_t* device_status_ptr();
int num_sms();

// ---------------------------------------------------------------- GEMM --------
// D[M, N] = X[M, K] . W^T + X2[M, R] . W2^T   (fp32 accumulate, one pass over D)
// W is K-major ([N, K] row-major) or MN-major ([K, N] row-major).
struct GemmArgs {
  const void* x;   // [M, K], row stride ldx
  const void* w;   // K-major: [N, K] stride ldw ; MN-major: [K, N] stride ldw
  const void* x2 = nullptr;  // [M, R64] stride ldx2 (nullptr when R == 0)
  const void* w2 = nullptr;  // K-major: [N, r] stride ldw2 ; MN-major: [r, N] stride ldw2
  void* d;         // [M, N] stride ldd
  const void* c = nullptr;  // optional addend [M, N] stride ldc, same type as d
  int64_t ldc = 0;
  const int32_t* c_index = nullptr;  // optional: addend row for output row m = c_index[m]
  int64_t c_rows = 0;                // rows of the addend table (bound for c_index)
  float acc_scale = 1.f;    // D = acc_scale * (X.W^T + X2.W2^T) + C
  // launched as a programmatic dependent of the previous kernel, which must
  // have written nothing this GEMM reads except X2 (waited for before X2 loads)
  bool overlap_prev = false;
  int64_t M, N, K;
  int64_t R = 0;   // extra reduction width, multiple of 16 (0 = none)
  int64_t w2_rows = 0;  // K-major: r (columns of w2); MN-major: r (rows of w2)
  int64_t ldx = 0, ldw = 0, ldx2 = 0, ldw2 = 0, ldd = 0;
  bool w_mn_major;
  Elt elt;
  int out_dtype;   // MLORA_DTYPE_*
};
int launch_gemm(const GemmArgs& a, cudaStream_t stream);

// ------------------------------------------------------ quantised GEMM ------
// D = X . deq(Wq)^T + X2 . up^T (forward, W K-major) or X . deq(Wq) + X2 . up
// (backward dx, W MN-major).  Wq rows/cols are the weight's [out, in] axes; the
// scales are pre-transposed to [groups, rows] (fp32 absmax or fp16 (scale,
// zero) pairs).  x, x2, up, d are bf16.
struct QGemmArgs {
  int scheme = 0;
  bool w_mn_major = false;
  const void* x = nullptr;
  const void* x2 = nullptr;
  const void* codes = nullptr;
  const void* scales_t = nullptr;
  const void* up = nullptr;  // forward: B [N, r] ; backward: A [r, K]
  void* d = nullptr;
  int64_t M = 0, N = 0, K = 0, R = 0;  // GEMM sizes (N = output columns, K = reduction)
  int64_t ldx = 0, ldx2 = 0, ldd = 0;
  int64_t group = 64;
  int64_t up_rows = 0, up_ld = 0, up_cols = 0;
};
int launch_qgemm(const QGemmArgs& a, cudaStream_t stream);

// ----------------------------------------------------------- decode (M <= 16) --
// y = x . deq(W)^T (+ B . sT^T) for at most 16 tokens; scheme 0 = dense bf16.
struct GemvArgs {
  int scheme = 0;
  const void* x = nullptr;         // bf16 [M, K]
  const void* w = nullptr;         // codes or bf16 weights, rows of the [N, K] weight
  const void* scales_t = nullptr;  // prepared scale table [G, prepared_ld(N)] (quantised)
  const void* b = nullptr;       // bf16 [N, r] or nullptr
  const float* st = nullptr;     // fp32 [rank_small_splits(K), M, r] partials of s.x.A^T
  void* y = nullptr;             // bf16 [M, N]
  float* partials = nullptr;     // [ctas, M, 128]: one partial row block per CTA, set to the
                                 // empty pattern by the kernel before (rank or fill kernel)
  int64_t M = 0, N = 0, K = 0, r = 0, group = 64;
  int64_t ldy = 0;  // row stride of y (0: N)
  bool pdl = false;  // launched as the programmatic dependent of the kernel before it
};
constexpr int64_t kGemvMaxTokens = 16;
// Decode launch shape: persistent CTAs (one per SM at most) over the stream-K
// unit range, ring depth, shared memory; split_blocks: some 128-row block is
// shared between CTAs (partials and flags needed).
struct DecodeConfig {
  int ctas;
  int stages;
  int smem;  // dynamic shared memory per CTA (bytes)
  bool split_blocks;
};
DecodeConfig decode_config(int scheme, int64_t M, int64_t N, int64_t K, int64_t r, int64_t group);
int64_t gemv_row_blocks(int64_t N);
int launch_gemv(const GemvArgs& a, cudaStream_t s);
int rank_small_splits(int64_t K);
// sT partials for the decode path; also sets the decode kernel's n_partials
// partial-slot floats (a multiple of 4) to their empty pattern.
int launch_rank_small(const void* x, const void* a, int64_t M, int64_t K, int64_t r, float scale,
                      float* st, float* partials, int64_t n_partials, cudaStream_t s);
// Sets n partial-slot floats to their empty pattern (decode without a rank
// kernel before it).
int launch_partials_fill(float* partials, int64_t n, cudaStream_t s);

// ------------------------------------------------------- rank projection -----
// out[m, j] = scale * sum_k X[m, k] * L[j, k] for j < R (L rows >= r are zero).
// Writes rows [M, ld_rows] (columns [R, ld_rows) zeroed) and/or the transpose
// [R, ld_t].  Split over K with a deterministic in-kernel reduction.
struct RankArgs {
  const void* x;   // [M, K] stride ldx
  const void* l;   // [r, K] stride ldl (rows r..R-1 read as zero)
  int64_t M, K, r, R;
  int64_t ldx, ldl;
  float scale;
  void* out_rows;  // bf16/f16 [M, ld_rows] or nullptr
  int64_t ld_rows;
  void* out_t;     // bf16/f16 [R, ld_t] or nullptr (ld_t >= M, multiple of 8)
  int64_t ld_t;
  // fp32 path: with split_out, out_rows row m = [part_0 | part_1 | part_2]
  // (R columns each) and out_t[j, s*M + m] = part_s, where part_s is the bf16
  // hi or lo part of the value as bit s of split_pattern says (0 = hi).
  bool split_out = false;
  // launched as a programmatic dependent of the kernel before it on the
  // stream: set-up overlaps that kernel, loads wait for it to finish
  bool overlap_prev = false;
  uint32_t split_pattern = 0;
  int splits;      // 1, 2, 4 or 8 (cluster size of the split reduction)
  Elt elt;
  // stacked adapters: row m keeps only columns [g*group_cols, (g+1)*group_cols)
  // of out_rows, g = row_group[m] (nullptr: all columns)
  const int32_t* row_group = nullptr;
  int64_t group_cols = 0;
};
int rank_splits(int64_t M, int64_t K);
int launch_rank(const RankArgs& a, cudaStream_t stream);

// ------------------------------------------------------- weight gradient -----
// out[p, j] = sum_m Big[m, p] * ST[j, m]   (p < P, j < r), optionally clipped,
// stored fp32 as out[p*ldo + j] (transposed = false) or out[j*ldo + p].
struct WgradArgs {
  const void* big;  // [M, P] stride ldb
  const void* st;   // [R, ld_st] (rows >= r are zero; ld_st >= M, multiple of 8)
  int64_t ld_st;
  int64_t M, P, r, R, ldb;
  float* out;
  int64_t ldo;
  bool transposed;
  bool accumulate = false;  // out += result (after the clip) instead of out = result
  bool out16 = false;       // out holds the operands' 16-bit type instead of fp32
  bool overlap_prev = false;  // programmatic dependent of the previous kernel
  float clip;       // <= 0: no clip
  int splits;       // 1, 2, 4 or 8 (cluster size of the split reduction)
  Elt elt;
};
int wgrad_splits(int64_t M, int64_t P, int nproblems);
int launch_wgrad(const WgradArgs* probs, int nprobs, cudaStream_t stream);

// ---------------------------------------------------------------- peers ------
// One-shot all-reduce over peer memory (see peer.cu); counter: one zeroed
// device word per communicator, reset by the kernel.
int launch_peer_allreduce(const void* bufs_dev, const void* flags_dev, int rank, int world,
                          uint32_t seq, float* out, int64_t n, float scale, uint32_t* counter,
                          cudaStream_t s);

// ------------------------------------------------------------ embedding ------
// g[t, :r] = B[idx[t]] ; gt[:R, t] = scale * B[idx[t]]^T (either may be null).
int launch_gather_rows(const int32_t* idx, const void* b, int64_t V, int64_t n_tok, int64_t r,
                       int64_t R, void* g, int64_t ldg, void* gt, int64_t ldgt, float scale,
                       Elt elt, cudaStream_t s);
// db[v] (+)= sum of u rows of the tokens with index v (sorted order; deterministic).
int launch_segment_rows(const int32_t* sorted_idx, const int32_t* order, const void* u,
                        int64_t ldu, int64_t n_tok, int64_t r, float* db, int64_t V,
                        bool accumulate, int dtype, cudaStream_t s);
int launch_embedding_f32(const int32_t* idx, const float* e, const float* a, const float* b,
                         float* out, int64_t n_tok, int64_t V, int64_t D, int64_t r, float scale,
                         cudaStream_t s);
int launch_rows_dot_f32(const float* dy, const float* a, float* u, int64_t n_tok, int64_t D,
                        int64_t r, float scale, cudaStream_t s);
int launch_embed_da_f32(const int32_t* idx, const float* b, const float* dy, float* da, int64_t V,
                        int64_t n_tok, int64_t D, int64_t r, float scale, bool accumulate,
                        cudaStream_t s);

// ---------------------------------------------------------- elementwise ------
int launch_transpose_pad(const void* b, int64_t N, int64_t r, int64_t ldb, void* bt, int64_t R,
                         Elt elt, cudaStream_t stream);

// Split-precision (bf16 hi/lo) copies of fp32 tensors; pattern bit s = 1 puts
// the lo part in segment s.  Patterns: kHHL = (hi, hi, lo), kHLH = (hi, lo, hi).
constexpr uint32_t kHHL = 0b100u;
constexpr uint32_t kHLH = 0b010u;
int launch_split3_cols(const float* src, int64_t rows, int64_t cols, int64_t ld_src, void* dst,
                       int64_t seg, int64_t ld_dst, uint32_t pattern, cudaStream_t stream);
int launch_split3_rows(const float* src, int64_t rows, int64_t cols, int64_t ld_src, void* dst,
                       int64_t seg_rows, uint32_t pattern, cudaStream_t stream);
int launch_split3_cols_t(const float* src, int64_t N, int64_t r, int64_t ld_src, void* dst,
                         int64_t R, int64_t seg, int64_t ld_dst, uint32_t pattern,
                         cudaStream_t stream);

// ------------------------------------------------------------- quantisation --
int launch_quantize(const void* w, int w_dtype, int64_t N, int64_t K, int scheme, int64_t g,
                    void* codes, void* scales, void* zeros, cudaStream_t s);
int launch_dequantize(int scheme, const void* codes, const void* scales, const void* zeros,
                      int64_t N, int64_t K, int64_t g, void* out, int out_dtype, cudaStream_t s);
// [rows, cols] -> [cols, ld] re-layouts (ld >= rows; padding columns zeroed).
int launch_transpose_f32(const float* src, int64_t rows, int64_t cols, int64_t ld, float* dst,
                         cudaStream_t s);
int launch_pack_scale_zero(const void* scales, const void* zeros, int64_t rows, int64_t cols,
                           int64_t ld, void* dst, cudaStream_t s);
// Row stride (elements) of the prepared scale table [groups, rows]: rows
// rounded up to 4 so every table row starts on a 16-byte boundary (TMA).
inline int64_t prepared_ld(int64_t rows) { return (rows + 3) / 4 * 4; }

// ---------------------------------------------------------------- optimizer --
int norm_grid();
int launch_grad_norm(const float* g, int64_t n, float max_norm, float* partials,
                     uint32_t* counter, float* out, cudaStream_t s);
int launch_adamw(void* param, int dtype, float* grad, float* m, float* v, const float* state,
                 int64_t n, float lr, float b1, float b2, float eps, float wd,
                 const float* grad_scale, int mode, cudaStream_t s);
int launch_adam_state_step(float* state, float b1, float b2, cudaStream_t s);

}  // namespace mlora
