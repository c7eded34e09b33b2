// One-shot all-reduce of a small fp32 buffer over NVLink peer memory (the
// LoRA gradients of a data-parallel step, ~0.5 MB per 4096x4096 rank-16
// layer).  Every rank's buffer and flag array live in symmetric memory (peer
// pointers from the caller).  One kernel per rank and step:
//   1. publish: make this rank's buffer visible system-wide, then raise its
//      flag in every peer's flag array to 2*seq-1;
//   2. block 0 alone waits (bounded) until all peers' flags in its own array
//      reach 2*seq-1 and records one go/abort verdict for the whole grid in
//      this GPU's counter words; the other CTAs wait for that verdict on a
//      local word (with back-off, so they do not load NVLink or L2 while a
//      kernel beside them computes).  With "go" every CTA sums the peers'
//      buffers in rank order -- the same operations on every rank, so the
//      results are bitwise identical; with "abort" no CTA writes `out`;
//   3. the last CTA to finish raises its flag in every peer to 2*seq and waits
//      for all peers to reach it: when the kernel has completed, no peer reads
//      this rank's buffer any more, so the caller may overwrite it.
// Flags only grow, so a peer already past a phase never blocks a slower one.
// A wait that exceeds 2 s records kDevPeerTimeout and gives up (no reduction).
// Peer data moves with plain (non-TMA) loads.
#include <string>

#include "internal.h"
#include "ptx.cuh"
#include "../../include/metallora_b200.h"

namespace mlora {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Waits until every mine[p] (p < world) is >= target (wrap-safe).  Bounded.
__device__ bool wait_flags(const uint32_t* mine, int world, uint32_t target, uint32_t* status) {
  const uint64_t t0 = globaltimer_ns();
  for (int p = 0; p < world; ++p) {
    uint32_t spins = 0;
    while (static_cast<int32_t>(ld_acquire_sys(mine + p) - target) < 0) {
      if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > MLORA_WAIT_BUDGET_NS) {
        record_status(status, kDevPeerTimeout);
        return false;
      }
    }
  }
  return true;
}

__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// counter words (this GPU's memory, zeroed once by the caller):
//   [0] CTAs done with this call (the last one resets it)
//   [1] seq of the latest verdict, [2] that verdict (1 = go, 0 = abort)
__global__ void __launch_bounds__(256) peer_allreduce_kernel(
    float* const* __restrict__ bufs, uint32_t* const* __restrict__ flags, int rank, int world,
    uint32_t seq, float* __restrict__ out, long long n, float scale, uint32_t* counter,
    uint32_t* status) {
  __shared__ int ok_s;
  __shared__ int last_s;
  const uint32_t t1 = 2u * seq - 1u, t2 = 2u * seq;
  const uint32_t* mine = flags[rank];
  if (blockIdx.x == 0) {
    if (threadIdx.x < world) {
      __threadfence_system();  // this rank's buffer, written by earlier kernels
      st_release_sys(flags[threadIdx.x] + rank, t1);
    }
    if (threadIdx.x == 0) {
      const int ok = wait_flags(mine, world, t1, status) ? 1 : 0;
      counter[2] = static_cast<uint32_t>(ok);
      st_release_gpu(counter + 1, seq);  // publishes the verdict word above
      ok_s = ok;
    }
  } else if (threadIdx.x == 0) {
    // block 0 decides within its own 2 s budget; this wait only bounds a
    // grid whose block 0 never ran
    const uint64_t t0 = globaltimer_ns();
    uint32_t ns = 32;
    int ok = 0;
    for (;;) {
      if (ld_acquire_gpu(counter + 1) == seq) {
        ok = static_cast<int>(__ldcg(counter + 2));
        break;
      }
      if (globaltimer_ns() - t0 > 2 * MLORA_WAIT_BUDGET_NS) {
        record_status(status, kDevPeerTimeout);
        break;
      }
      __nanosleep(ns);
      if (ns < 1024) ns *= 2;
    }
    ok_s = ok;
  }
  __syncthreads();
  if (ok_s) {
    const long long n4 = n / 4;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += stride) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int p = 0; p < world; ++p) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(bufs[p]) + i);  // at the peer's L2
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      reinterpret_cast<float4*>(out)[i] =
          make_float4(acc.x * scale, acc.y * scale, acc.z * scale, acc.w * scale);
    }
    for (long long i = n4 * 4 + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
         i < n; i += stride) {
      float acc = 0.f;
      for (int p = 0; p < world; ++p) acc += __ldcg(bufs[p] + i);
      out[i] = acc * scale;
    }
  }
  __syncthreads();  // this CTA's peer loads have all been consumed
  if (threadIdx.x == 0) {
    __threadfence();
    last_s = atomicAdd(counter, 1u) == gridDim.x - 1 ? 1 : 0;
  }
  __syncthreads();
  if (!last_s) return;
  if (threadIdx.x == 0) *counter = 0;  // ready for the next call
  if (threadIdx.x < world) {
    __threadfence_system();
    st_release_sys(flags[threadIdx.x] + rank, t2);
  }
  __syncthreads();
  if (threadIdx.x == 0) wait_flags(mine, world, t2, status);
}

}  // namespace

int launch_peer_allreduce(const void* bufs_dev, const void* flags_dev, int rank, int world,
                          uint32_t seq, float* out, int64_t n, float scale, uint32_t* counter,
                          cudaStream_t s) {
  LaunchScope scope(kKindOptim, s);
  int64_t blocks = (n / 4 + 255) / 256;
  if (blocks < 1) blocks = 1;
  if (blocks > num_sms()) blocks = num_sms();  // all CTAs resident: flag waits cannot starve
  peer_allreduce_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
      static_cast<float* const*>(bufs_dev), static_cast<uint32_t* const*>(flags_dev), rank, world,
      seq, out, n, scale, counter, device_status_ptr());
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("peer_allreduce launch: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

}  // namespace mlora
