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

}  // namespace

int launch_transpose_pad(const void* b, int64_t N, int64_t r, int64_t ldb, void* bt, int64_t R,
                         Elt elt, cudaStream_t stream) {
  dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>((R + 31) / 32));
  dim3 block(32, 8);
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
