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

// Per-device cache of the array's device address, valid for the context it
// was looked up in.  Host code only sees a host-side stand-in for the symbol;
// the real address comes from the runtime with the device current.  The cache
// is keyed on the driver's unique context id, so a context torn down and
// re-created (cudaDeviceReset) gets a fresh lookup instead of a stale address,
// and only successful lookups are kept: a failed one is retried on the next
// call.
struct ScratchSlot {
  std::mutex mu;
  unsigned long long ctx_id = 0;
  bool valid = false;
  void* ptr = nullptr;
};
ScratchSlot g_slot[kMaxDevices];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current context (0 when it cannot be read;
// the address is then looked up again on every call).
unsigned long long current_context_id() {
  static std::once_flag once;
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (get_current == nullptr || get_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of the scratch array on `device` (which is current).
void* scratch_address(int device, cudaError_t* err) {
  ScratchSlot& slot = g_slot[device];
  std::lock_guard<std::mutex> lock(slot.mu);
  const unsigned long long id = current_context_id();
  if (slot.valid && id != 0 && slot.ctx_id == id) {
    *err = cudaSuccess;
    return slot.ptr;
  }
  void* p = nullptr;
  *err = cudaGetSymbolAddress(&p, g_lora_grad_scratch);
  if (*err != cudaSuccess || p == nullptr) {
    cudaGetLastError();  // not sticky: the next call tries again
    slot.valid = false;
    return nullptr;
  }
  slot.ptr = p;
  slot.ctx_id = id;
  slot.valid = id != 0;
  return p;
}

}  // namespace

extern "C" {

size_t mlora_lora_grads_static_scratch_bytes(void) { return kStaticScratchBytes; }

int mlora_lora_grads_static(const void* dy, const void* x, const void* a, const void* b,
                            float* da, float* db, int64_t M, int64_t K, int64_t N, int64_t r,
                            float alpha, float clip_value, int dtype, void* stream) {
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
  if (e != cudaSuccess) {
    mlora::set_error(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  if (device < 0 || device >= kMaxDevices) {
    mlora::set_error("mlora_lora_grads_static: device index " + std::to_string(device) +
                     " exceeds the " + std::to_string(kMaxDevices) +
                     "-device limit of the built-in scratch");
    return MLORA_ERR_UNSUPPORTED;
  }
  void* scratch = scratch_address(device, &e);
  if (scratch == nullptr) {
    mlora::set_error(std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  // Same computation as mlora_lora_backward without dx.
  return mlora_lora_backward(dy, x, nullptr, a, b, nullptr, nullptr, da, db, M, K, N, r, alpha,
                             clip_value, dtype, scratch, kStaticScratchBytes, stream);
}

}  // extern "C"
