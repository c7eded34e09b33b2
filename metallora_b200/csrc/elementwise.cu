// Bandwidth-bound helper kernels of the LoRA path.
#include "internal.h"
#include "ptx.cuh"
#include "../../include/metallora_b200.h"

namespace mlora {
namespace {

// bt[j, n] = b[n, j] for j < r, 0 for r <= j < R.  b is [N, r] with row stride ldb.
template <typename T>
__global__ void transpose_pad_kernel(const T* __restrict__ b, int64_t N, int64_t r, int64_t ldb,
                                     T* __restrict__ bt, int64_t R) {
  // the rank projection that follows may start its set-up now
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ T tile[32][33];
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int64_t j0 = static_cast<int64_t>(blockIdx.y) * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t n = n0 + i, j = j0 + threadIdx.x;
    tile[i][threadIdx.x] = (n < N && j < r) ? b[n * ldb + j] : T(0.f);
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t j = j0 + i, n = n0 + threadIdx.x;
    if (j < R && n < N) bt[j * N + n] = tile[threadIdx.x][i];
  }
}

// Split-precision copies for the fp32 path.  A float v is written as the
// bf16 pair hi = rn(v), lo = rn(v - hi); hi*hi' + hi*lo' + lo*hi' reproduces
// a product of two fp32 values to ~2^-16 relative.  `pattern` bit s selects lo
// for segment s (0 = hi).

// dst[row, s*seg + c] = part_s(src[row, c]) for c < cols, 0 for cols <= c < seg.
__global__ void split3_cols_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                                   int64_t ld_src, __nv_bfloat16* __restrict__ dst, int64_t seg,
                                   int64_t ld_dst, uint32_t pattern) {
  const int64_t total = rows * seg;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / seg, c = i % seg;
    const float v = c < cols ? src[row * ld_src + c] : 0.f;
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
    __nv_bfloat16* d = dst + row * ld_dst + c;
#pragma unroll
    for (int s = 0; s < 3; ++s) d[s * seg] = ((pattern >> s) & 1u) ? lo : hi;
  }
}

// dst[s*seg_rows + row, c] = part_s(src[row, c]) for row < rows, 0 for rows <= row < seg_rows.
__global__ void split3_rows_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                                   int64_t ld_src, __nv_bfloat16* __restrict__ dst,
                                   int64_t seg_rows, uint32_t pattern) {
  const int64_t total = seg_rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / cols, c = i % cols;
    const float v = row < rows ? src[row * ld_src + c] : 0.f;
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
#pragma unroll
    for (int s = 0; s < 3; ++s)
      dst[(s * seg_rows + row) * cols + c] = ((pattern >> s) & 1u) ? lo : hi;
  }
}

// dst[j, s*seg + n] = part_s(src[n, j]) for j < r, 0 for r <= j < R:
// transpose of src [N, r] into segments of width seg (>= N) per row.
__global__ void split3_cols_t_kernel(const float* __restrict__ src, int64_t N, int64_t r,
                                     int64_t ld_src, __nv_bfloat16* __restrict__ dst, int64_t R,
                                     int64_t seg, int64_t ld_dst, uint32_t pattern) {
  const int64_t total = R * N;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t j = i / N, n = i % N;
    const float v = j < r ? src[n * ld_src + j] : 0.f;
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
#pragma unroll
    for (int s = 0; s < 3; ++s) dst[j * ld_dst + s * seg + n] = ((pattern >> s) & 1u) ? lo : hi;
  }
}

int grid_for(int64_t total) {
  int64_t g = (total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  return static_cast<int>(g < cap ? (g > 0 ? g : 1) : cap);
}

int launch_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

}  // namespace

int launch_split3_cols(const float* src, int64_t rows, int64_t cols, int64_t ld_src, void* dst,
                       int64_t seg, int64_t ld_dst, uint32_t pattern, cudaStream_t stream) {
  LaunchScope scope(kKindElementwise, stream);
  split3_cols_kernel<<<grid_for(rows * seg), 256, 0, stream>>>(
      src, rows, cols, ld_src, static_cast<__nv_bfloat16*>(dst), seg, ld_dst, pattern);
  return launch_check("split3_cols");
}

int launch_split3_rows(const float* src, int64_t rows, int64_t cols, int64_t ld_src, void* dst,
                       int64_t seg_rows, uint32_t pattern, cudaStream_t stream) {
  LaunchScope scope(kKindElementwise, stream);
  split3_rows_kernel<<<grid_for(seg_rows * cols), 256, 0, stream>>>(
      src, rows, cols, ld_src, static_cast<__nv_bfloat16*>(dst), seg_rows, pattern);
  return launch_check("split3_rows");
}

int launch_split3_cols_t(const float* src, int64_t N, int64_t r, int64_t ld_src, void* dst,
                         int64_t R, int64_t seg, int64_t ld_dst, uint32_t pattern,
                         cudaStream_t stream) {
  LaunchScope scope(kKindElementwise, stream);
  split3_cols_t_kernel<<<grid_for(R * N), 256, 0, stream>>>(
      src, N, r, ld_src, static_cast<__nv_bfloat16*>(dst), R, seg, ld_dst, pattern);
  return launch_check("split3_cols_t");
}

int launch_transpose_pad(const void* b, int64_t N, int64_t r, int64_t ldb, void* bt, int64_t R,
                         Elt elt, cudaStream_t stream) {
  dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>((R + 31) / 32));
  dim3 block(32, 8);
  LaunchScope scope(kKindElementwise, stream);
  if (elt == Elt::kBF16)
    transpose_pad_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(b), N, r, ldb, static_cast<__nv_bfloat16*>(bt), R);
  else
    transpose_pad_kernel<__half><<<grid, block, 0, stream>>>(static_cast<const __half*>(b), N, r,
                                                             ldb, static_cast<__half*>(bt), R);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("transpose launch: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

}  // namespace mlora
