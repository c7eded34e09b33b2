// Optimizer kernels of the LoRA training step (reference: the live AdamW kernel
// python/metal_lora/kernels.py:314-344, its step-state kernel :351-362, and the
// global-norm clip of trainer.py:237-240).  They run over flat buffers: all
// LoRA A/B factors of a model live in one contiguous fp32 array, so one launch
// updates every adapter.
#include <string>

#include "internal.h"
#include "ptx.cuh"
#include "../../include/metallora_b200.h"

namespace mlora {
namespace {

constexpr int kNormThreads = 256;

// Sum of squares of g[0..n): one fp32 partial per CTA (grid-stride, fixed grid),
// then the last CTA to finish adds the partials in CTA order -- deterministic
// for a given grid size.  out[0] = clip scale min(1, max_norm / (norm + 1e-6))
// (1 when max_norm <= 0), out[1] = norm.
__global__ void __launch_bounds__(kNormThreads)
    grad_norm_kernel(const float* __restrict__ g, int64_t n, float max_norm, float* partials,
                     uint32_t* counter, float* out) {
  __shared__ float red[kNormThreads / 32];
  __shared__ bool last;
  float s = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = g[i];
    s = fmaf(v, v, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kNormThreads / 32; ++w) t += red[w];
    partials[blockIdx.x] = t;
    __threadfence();
    const uint32_t ticket = atomicAdd(counter, 1u);
    last = ticket == gridDim.x - 1;
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  float total = 0.f;
  for (unsigned b = 0; b < gridDim.x; ++b) total += __ldcg(partials + b);
  const float norm = sqrtf(total);
  out[1] = norm;
  out[0] = max_norm > 0.f ? fminf(1.f, max_norm / (norm + 1e-6f)) : 1.f;
  *counter = 0;
}

// AdamW with bias correction in the live kernel's operation order
// (kernels.py:330-343).  state = [step, beta1^step, beta2^step] on the device.
// The gradient is read once (times *grad_scale when given) and zeroed, as the
// reference kernel does.  mode 1 = SGD (p -= lr * g).
template <typename P>
__global__ void adamw_kernel(P* __restrict__ param, float* __restrict__ grad, float* __restrict__ m,
                             float* __restrict__ v, const float* __restrict__ state, int64_t n,
                             float lr, float b1, float b2, float eps, float wd,
                             const float* __restrict__ grad_scale, int mode) {
  const float gs = grad_scale != nullptr ? *grad_scale : 1.f;
  const float b1t = mode == 0 ? state[1] : 0.f;
  const float b2t = mode == 0 ? state[2] : 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    // Explicitly rounded operations (no FMA contraction) keep every value
    // identical to the reference kernel's operation order.
    const float g = __fmul_rn(grad[i], gs);
    grad[i] = 0.f;
    float p = static_cast<float>(param[i]);
    if (mode == 1) {
      p = __fsub_rn(p, __fmul_rn(lr, g));
    } else {
      const float m_val = __fadd_rn(__fmul_rn(b1, m[i]), __fmul_rn(__fsub_rn(1.0f, b1), g));
      const float v_val =
          __fadd_rn(__fmul_rn(b2, v[i]), __fmul_rn(__fmul_rn(__fsub_rn(1.0f, b2), g), g));
      m[i] = m_val;
      v[i] = v_val;
      const float m_hat = __fdiv_rn(m_val, __fsub_rn(1.0f, b1t));
      const float v_hat = __fdiv_rn(v_val, __fsub_rn(1.0f, b2t));
      const float upd = __fadd_rn(__fdiv_rn(m_hat, __fadd_rn(__fsqrt_rn(v_hat), eps)),
                                  __fmul_rn(wd, p));
      p = __fsub_rn(p, __fmul_rn(lr, upd));
    }
    param[i] = static_cast<P>(p);
  }
}

// kernels.py:355-361: step += 1; beta powers *= beta.
__global__ void adam_state_step_kernel(float* state, float b1, float b2) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    state[0] += 1.0f;
    state[1] *= b1;
    state[2] *= b2;
  }
}

int grid_cap(int64_t n, int per_block) {
  int64_t g = (n + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  if (g > cap) g = cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

}  // namespace

int norm_grid() { return 2 * num_sms(); }

int launch_grad_norm(const float* g, int64_t n, float max_norm, float* partials,
                     uint32_t* counter, float* out, cudaStream_t s) {
  LaunchScope scope(kKindOptim, s);
  grad_norm_kernel<<<norm_grid(), kNormThreads, 0, s>>>(g, n, max_norm, partials, counter, out);
  return check_launch("grad_norm");
}

int launch_adamw(void* param, int dtype, float* grad, float* m, float* v, const float* state,
                 int64_t n, float lr, float b1, float b2, float eps, float wd,
                 const float* grad_scale, int mode, cudaStream_t s) {
  LaunchScope scope(kKindOptim, s);
  const int grid = grid_cap(n, 256);
  if (dtype == MLORA_DTYPE_F32)
    adamw_kernel<float><<<grid, 256, 0, s>>>(static_cast<float*>(param), grad, m, v, state, n, lr,
                                             b1, b2, eps, wd, grad_scale, mode);
  else if (dtype == MLORA_DTYPE_BF16)
    adamw_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<__nv_bfloat16*>(param), grad, m,
                                                     v, state, n, lr, b1, b2, eps, wd, grad_scale,
                                                     mode);
  else
    adamw_kernel<__half><<<grid, 256, 0, s>>>(static_cast<__half*>(param), grad, m, v, state, n,
                                              lr, b1, b2, eps, wd, grad_scale, mode);
  return check_launch("adamw");
}

int launch_adam_state_step(float* state, float b1, float b2, cudaStream_t s) {
  LaunchScope scope(kKindOptim, s);
  adam_state_step_kernel<<<1, 32, 0, s>>>(state, b1, b2);
  return check_launch("adam_state_step");
}

}  // namespace mlora
