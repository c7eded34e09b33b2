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
  const void* x2;  // [M, R64] stride ldx2 (nullptr when R == 0)
  const void* w2;  // K-major: [N, r] stride ldw2 ; MN-major: [r, N] stride ldw2
  void* d;         // [M, N] stride ldd
  int64_t M, N, K;
  int64_t R;       // extra reduction width, multiple of 16 (0 = none)
  int64_t w2_rows; // K-major: r (columns of w2); MN-major: r (rows of w2)
  int64_t ldx, ldw, ldx2, ldw2, ldd;
  bool w_mn_major;
  Elt elt;
  int out_dtype;   // MLORA_DTYPE_*
};
int launch_gemm(const GemmArgs& a, cudaStream_t stream);

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
  float* partials; // [splits, M, R] fp32 workspace
  uint32_t* counters;  // [ceil(M/128)] zeroed
  int splits;
  Elt elt;
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
  float clip;       // <= 0: no clip
  float* partials;  // [splits, P, R]
  uint32_t* counters;  // [ceil(P/128)] zeroed
  int splits;
  Elt elt;
};
int wgrad_splits(int64_t M, int64_t P, int nproblems);
int launch_wgrad(const WgradArgs* probs, int nprobs, cudaStream_t stream);

// ---------------------------------------------------------- elementwise ------
int launch_transpose_pad(const void* b, int64_t N, int64_t r, int64_t ldb, void* bt, int64_t R,
                         Elt elt, cudaStream_t stream);

}  // namespace mlora
