// LoRA embedding (python/metal_lora/layers.py:194-230):
//   out[t, :] = E[idx[t], :] + s * B[idx[t], :] . A          (s = alpha / r)
// bf16/fp16: the gathered B rows are the A operand of the tcgen05 GEMM (K = r),
// A is read MN-major, and E's rows are gathered into the epilogue addend; the
// gradients come from the rank kernel (U = s dy.A^T), a deterministic segment
// sum of U over tokens sorted by index (dB), and the weight-gradient kernel
// (dA = s B[idx]^T . dy).  fp32 runs the same math on CUDA cores.
// An index outside [0, V) contributes nothing and is reported in the device
// status word (kDevBadIndex).
#include <string>

#include "internal.h"
#include "ptx.cuh"
#include "../../include/metallora_b200.h"

namespace mlora {
namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v) { return static_cast<float>(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v) { return static_cast<T>(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// g[t, j] = B[idx[t], j] (j < r, row stride ldg); gt[j, t] = scale * B[idx[t], j]
// for j < R (zero for r <= j < R; row stride ldgt).  Either output may be null.
template <typename T>
__global__ void gather_rows_kernel(const int32_t* __restrict__ idx, const T* __restrict__ b,
                                   int64_t V, int64_t n_tok, int r, int R, T* __restrict__ g,
                                   int64_t ldg, T* __restrict__ gt, int64_t ldgt, float scale,
                                   uint32_t* status) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= n_tok * R) return;
  const int64_t t = e / R;
  const int j = static_cast<int>(e % R);
  const int64_t v = idx[t];
  float val = 0.f;
  if (v < 0 || v >= V) {
    if (j == 0) record_status(status, kDevBadIndex);
  } else if (j < r) {
    val = to_f(b[v * r + j]);
  }
  if (g != nullptr && j < r) g[t * ldg + j] = from_f<T>(val);
  if (gt != nullptr) gt[static_cast<int64_t>(j) * ldgt + t] = from_f<T>(val * scale);
}

// db[v, j] (+)= sum of u[order[q], j] over the run of sorted_idx equal to v, in
// sorted (stable: token) order.  One thread per (sorted position, j); only run
// starts work, so every db row is written by exactly one thread per column.
template <typename T>
__global__ void segment_rows_kernel(const int32_t* __restrict__ sorted_idx,
                                    const int32_t* __restrict__ order, const T* __restrict__ u,
                                    int64_t ldu, int64_t n_tok, int r, float* __restrict__ db,
                                    int64_t V, int accumulate, uint32_t* status) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= n_tok * r) return;
  const int64_t p = e / r;
  const int j = static_cast<int>(e % r);
  const int v = sorted_idx[p];
  if (p > 0 && sorted_idx[p - 1] == v) return;
  if (v < 0 || v >= V) {
    if (j == 0) record_status(status, kDevBadIndex);
    return;
  }
  float acc = 0.f;
  for (int64_t q = p; q < n_tok && sorted_idx[q] == v; ++q)
    acc += to_f(u[static_cast<int64_t>(order[q]) * ldu + j]);
  float* dst = db + static_cast<int64_t>(v) * r + j;
  *dst = accumulate ? *dst + acc : acc;
}

// fp32 forward: one CTA per token; the token's B row in shared memory.
__global__ void embedding_f32_kernel(const int32_t* __restrict__ idx, const float* __restrict__ e,
                                     const float* __restrict__ a, const float* __restrict__ b,
                                     float* __restrict__ out, int64_t V, int64_t D, int r,
                                     float scale, uint32_t* status) {
  __shared__ float brow[256];
  const int64_t t = blockIdx.x;
  const int64_t v = idx[t];
  const bool ok = v >= 0 && v < V;
  if (!ok && threadIdx.x == 0) record_status(status, kDevBadIndex);
  for (int j = threadIdx.x; j < r; j += blockDim.x) brow[j] = ok ? b[v * r + j] : 0.f;
  __syncthreads();
  for (int64_t d = threadIdx.x; d < D; d += blockDim.x) {
    float lora = 0.f;
    for (int j = 0; j < r; ++j) lora = fmaf(brow[j], a[static_cast<int64_t>(j) * D + d], lora);
    out[t * D + d] = ok ? e[v * D + d] + scale * lora : 0.f;
  }
}

// fp32 U = scale * dy . A^T: one CTA per token, one warp per rank column.
__global__ void rows_dot_f32_kernel(const float* __restrict__ dy, const float* __restrict__ a,
                                    float* __restrict__ u, int64_t D, int r, float scale) {
  const int64_t t = blockIdx.x;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j = w; j < r; j += blockDim.x >> 5) {
    float acc = 0.f;
    for (int64_t d = lane; d < D; d += 32) acc = fmaf(dy[t * D + d], a[static_cast<int64_t>(j) * D + d], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) u[t * r + j] = acc * scale;
  }
}

// fp32 dA[j, d] (+)= scale * sum_t B[idx[t], j] dy[t, d], tokens in order.
__global__ void embed_da_f32_kernel(const int32_t* __restrict__ idx, const float* __restrict__ b,
                                    const float* __restrict__ dy, float* __restrict__ da,
                                    int64_t V, int64_t n_tok, int64_t D, int r, float scale,
                                    int accumulate) {
  const int64_t d = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int j = blockIdx.y;
  if (d >= D) return;
  float acc = 0.f;
  for (int64_t t = 0; t < n_tok; ++t) {
    const int64_t v = idx[t];
    if (v >= 0 && v < V) acc = fmaf(b[v * r + j], dy[t * D + d], acc);
  }
  float* dst = da + static_cast<int64_t>(j) * D + d;
  *dst = accumulate ? *dst + acc * scale : acc * scale;
}

int launched(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

unsigned blocks_for(int64_t n, int threads) {
  return static_cast<unsigned>((n + threads - 1) / threads);
}

}  // namespace

int launch_gather_rows(const int32_t* idx, const void* b, int64_t V, int64_t n_tok, int64_t r,
                       int64_t R, void* g, int64_t ldg, void* gt, int64_t ldgt, float scale,
                       Elt elt, cudaStream_t s) {
  LaunchScope scope(kKindElementwise, s);
  const unsigned grid = blocks_for(n_tok * R, 256);
  if (elt == Elt::kBF16)
    gather_rows_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        idx, static_cast<const __nv_bfloat16*>(b), V, n_tok, static_cast<int>(r),
        static_cast<int>(R), static_cast<__nv_bfloat16*>(g), ldg, static_cast<__nv_bfloat16*>(gt),
        ldgt, scale, device_status_ptr());
  else
    gather_rows_kernel<__half><<<grid, 256, 0, s>>>(
        idx, static_cast<const __half*>(b), V, n_tok, static_cast<int>(r), static_cast<int>(R),
        static_cast<__half*>(g), ldg, static_cast<__half*>(gt), ldgt, scale, device_status_ptr());
  return launched("gather_rows");
}

int launch_segment_rows(const int32_t* sorted_idx, const int32_t* order, const void* u,
                        int64_t ldu, int64_t n_tok, int64_t r, float* db, int64_t V,
                        bool accumulate, int dtype, cudaStream_t s) {
  LaunchScope scope(kKindElementwise, s);
  const unsigned grid = blocks_for(n_tok * r, 256);
  const int acc = accumulate ? 1 : 0;
  if (dtype == MLORA_DTYPE_BF16)
    segment_rows_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        sorted_idx, order, static_cast<const __nv_bfloat16*>(u), ldu, n_tok, static_cast<int>(r),
        db, V, acc, device_status_ptr());
  else if (dtype == MLORA_DTYPE_F16)
    segment_rows_kernel<__half><<<grid, 256, 0, s>>>(sorted_idx, order,
                                                     static_cast<const __half*>(u), ldu, n_tok,
                                                     static_cast<int>(r), db, V, acc,
                                                     device_status_ptr());
  else
    segment_rows_kernel<float><<<grid, 256, 0, s>>>(sorted_idx, order, static_cast<const float*>(u),
                                                    ldu, n_tok, static_cast<int>(r), db, V, acc,
                                                    device_status_ptr());
  return launched("segment_rows");
}

int launch_embedding_f32(const int32_t* idx, const float* e, const float* a, const float* b,
                         float* out, int64_t n_tok, int64_t V, int64_t D, int64_t r, float scale,
                         cudaStream_t s) {
  LaunchScope scope(kKindElementwise, s);
  embedding_f32_kernel<<<static_cast<unsigned>(n_tok), 256, 0, s>>>(
      idx, e, a, b, out, V, D, static_cast<int>(r), scale, device_status_ptr());
  return launched("embedding_f32");
}

int launch_rows_dot_f32(const float* dy, const float* a, float* u, int64_t n_tok, int64_t D,
                        int64_t r, float scale, cudaStream_t s) {
  LaunchScope scope(kKindElementwise, s);
  rows_dot_f32_kernel<<<static_cast<unsigned>(n_tok), 256, 0, s>>>(dy, a, u, D,
                                                                   static_cast<int>(r), scale);
  return launched("rows_dot_f32");
}

int launch_embed_da_f32(const int32_t* idx, const float* b, const float* dy, float* da, int64_t V,
                        int64_t n_tok, int64_t D, int64_t r, float scale, bool accumulate,
                        cudaStream_t s) {
  LaunchScope scope(kKindElementwise, s);
  dim3 grid(blocks_for(D, 256), static_cast<unsigned>(r));
  embed_da_f32_kernel<<<grid, 256, 0, s>>>(idx, b, dy, da, V, n_tok, D, static_cast<int>(r), scale,
                                           accumulate ? 1 : 0);
  return launched("embed_da_f32");
}

}  // namespace mlora
