// Allocation-free variant of the LoRA weight-gradient entry point.
//
// mlora_lora_backward needs scratch (the transposed B and the rank
// intermediates s.dy.B and s.x.A^T) and takes it
// from a workspace the caller allocates.  Some callers cannot allocate device
// memory when they run the backward: a process that hands all device memory to
// its own pool at start-up and has none left to give, or a latency-critical
// loop that must not call cudaMalloc because it can wait on the whole device
// and stall every stream.  This entry point serves them with a fixed scratch
// array that lives in the library itself (a static __device__ array, present
// on every GPU that loads the library until the process exits).
#include <mutex>
#include <string>

#include "internal.h"
#include "../../include/metallora_b200.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;  // 32 MiB per device

// Scratch shared by every call on a device; calls keep no state in it between
// them except what each call clears itself.
static __device__ __align__(256) unsigned char g_lora_grad_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::once_flag g_setup_once[kMaxDevices];
void* g_scratch_ptr[kMaxDevices] = {};
cudaError_t g_setup_err[kMaxDevices] = {};

// Device address of the scratch array for the current device (host code only
// sees a host-side stand-in for the symbol; the real address comes from the
// runtime, once per device, with that device current).
void* scratch_address(int device, cudaError_t* err) {
  std::call_once(g_setup_once[device], [device]() {
    void* p = nullptr;
    g_setup_err[device] = cudaGetSymbolAddress(&p, g_lora_grad_scratch);
    g_scratch_ptr[device] = (g_setup_err[device] == cudaSuccess) ? p : nullptr;
  });
  *err = g_setup_err[device];
  return g_scratch_ptr[device];
}

}  // namespace

extern "C" {

size_t mlora_lora_grads_static_scratch_bytes(void) { return kStaticScratchBytes; }

int mlora_lora_grads_static(const void* dy, const void* x, const void* a, const void* b, float* da,
                            float* db, int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                            float clip_value, int dtype, void* stream) {
  if (dtype != MLORA_DTYPE_BF16 && dtype != MLORA_DTYPE_F16) {
    mlora::set_error("mlora_lora_grads_static takes BF16 or F16 inputs");
    return MLORA_ERR_UNSUPPORTED;
  }
  const size_t need = mlora_lora_backward_workspace_bytes(M, K, N, r, dtype);
  if (need == 0) {
    mlora::set_error("M, K, N and r must be positive");
    return MLORA_ERR_INVALID_ARG;
  }
  if (need > kStaticScratchBytes) {
    mlora::set_error("mlora_lora_grads_static: this shape needs " + std::to_string(need) +
                     " bytes of scratch; the built-in array holds " +
                     std::to_string(kStaticScratchBytes) +
                     " (use mlora_lora_backward with a workspace)");
    return MLORA_ERR_WORKSPACE;
  }
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess || device < 0 || device >= kMaxDevices) {
    mlora::set_error(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  void* scratch = scratch_address(device, &e);
  if (e != cudaSuccess || scratch == nullptr) {
    mlora::set_error(std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  // Same computation as mlora_lora_backward without dx.
  return mlora_lora_backward(dy, x, nullptr, a, b, nullptr, nullptr, da, db, M, K, N, r, alpha,
                             clip_value, dtype, scratch, kStaticScratchBytes, stream);
}

}  // extern "C"
