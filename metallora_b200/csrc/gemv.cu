// Decode-size LoRA linear (M <= 16 tokens): HBM-bound on the base weight.
//
//   sT[m, j] = s * sum_k x[m, k] A[j, k]                        (lora_rank_small_kernel)
//   y[m, n]  = sum_k deq(W[n, k]) x[m, k] + sum_j B[n, j] sT[m, j]   (lora_gemv_kernel)
//
// The weight is streamed once with 128-bit loads by warps that each own 32
// output rows; every lane dequantises the 32 consecutive weights it loaded
// (bf16_rn of the fp32 reference dequant, as the tensor-core paths) straight
// into the B fragments of mma.m16n8k16 (the 16 tokens are the A operand, read
// from shared memory).  The in-feature axis is split across CTAs; fp32 partial
// tiles go to a workspace and the last CTA of each row block adds them in split
// order (deterministic), adds the rank-r term and writes y.
//
// Fragment order: lane (g = lane/4, q = lane%4) loads weights k in [32q, 32q+32)
// of a 128-wide chunk of row n0 + g.  In MMA block b (0..7) its k-slots
// {2q, 2q+1} hold k = 32q+4b+{0,1} and {2q+8, 2q+9} hold k = 32q+4b+{2,3}; the
// token fragments use the same permutation, which leaves the dot products
// unchanged.
#include <string>

#include "internal.h"
#include "ptx.cuh"
#include "quant.cuh"
#include "../../include/metallora_b200.h"

namespace mlora {
namespace {

constexpr int kGemvWarps = 8;
constexpr int kRG = 2;                                 // row groups (of 8 rows) per warp
constexpr int kRowsPerWarp = 8 * kRG;
constexpr int kRowsPerCta = kGemvWarps * kRowsPerWarp;  // 128
constexpr int kChunk = 128;                            // k per chunk
constexpr int kMaxTok = 16;
constexpr int kXPad = 8;  // bf16 elements of padding per staged token row

// scheme: 0 = dense bf16, else QuantScheme.
template <int kScheme>
struct GemvTraits {
  static constexpr int kBitsPerW = kScheme == 0 ? 16 : (kScheme == kINT8 ? 8 : 4);
  static constexpr int kLoads = kBitsPerW * 32 / 128;  // 16-byte loads per lane per row group
};

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 32 consecutive weights of one row, loaded as raw words, -> 16 packed bf16x2
// (pairs k, k+1 for k = 0, 2, ..., 30 of the lane's span).
template <int kScheme>
__device__ __forceinline__ void to_bf16_pairs(const uint4 (&raw)[GemvTraits<kScheme>::kLoads],
                                              float s, float z, const float* lut,
                                              uint32_t (&out)[16]) {
  if constexpr (kScheme == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      out[4 * i + 0] = raw[i].x;
      out[4 * i + 1] = raw[i].y;
      out[4 * i + 2] = raw[i].z;
      out[4 * i + 3] = raw[i].w;
    }
  } else if constexpr (kScheme == kINT8) {
    const uint32_t w[8] = {raw[0].x, raw[0].y, raw[0].z, raw[0].w,
                           raw[1].x, raw[1].y, raw[1].z, raw[1].w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      out[2 * i] = pack2<__nv_bfloat16>(dequant_int(w[i] & 0xFFu, s, z),
                                        dequant_int((w[i] >> 8) & 0xFFu, s, z));
      out[2 * i + 1] = pack2<__nv_bfloat16>(dequant_int((w[i] >> 16) & 0xFFu, s, z),
                                            dequant_int(w[i] >> 24, s, z));
    }
  } else {
    const uint32_t w[4] = {raw[0].x, raw[0].y, raw[0].z, raw[0].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint32_t c0 = (w[i] >> (8 * h)) & 0xFu, c1 = (w[i] >> (8 * h + 4)) & 0xFu;
        float v0, v1;
        if constexpr (kScheme == kNF4) {
          v0 = dequant_nf4(c0, s, lut);
          v1 = dequant_nf4(c1, s, lut);
        } else {
          v0 = dequant_int(c0, s, z);
          v1 = dequant_int(c1, s, z);
        }
        out[4 * i + h] = pack2<__nv_bfloat16>(v0, v1);
      }
    }
  }
}

struct GemvParams {
  const __nv_bfloat16* x;   // [M, K]
  const uint8_t* w;         // codes (or bf16 weights) [N, row_bytes]
  const void* scales;       // NF4: fp32 [N, G]; INT: fp16 [N, G]
  const __half* zeros;      // INT: fp16 [N, G]
  const __nv_bfloat16* b;   // [N, r] (nullptr: no rank term)
  const float* st;          // [st_splits, M, r] fp32 partial sums of s.x.A^T
  int st_splits;
  __nv_bfloat16* y;         // [M, N]
  float* partials;          // [splits, M, N]
  uint32_t* counters;       // [gemv_row_blocks(N)]
  int M, N, K, r, group, splits, k_per_split;
  long long row_bytes;
  uint32_t* status;
};

template <int kScheme>
__global__ void __launch_bounds__(kGemvWarps * 32, 3) lora_gemv_kernel(const GemvParams p) {
  using Tr = GemvTraits<kScheme>;
  extern __shared__ __align__(16) uint8_t smem_g[];
  __shared__ float lut[16];
  __shared__ uint32_t last_flag;
  const int kspan = p.k_per_split;
  const int xld = kspan + kXPad;  // bf16 per staged token row
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_g);

  const int rb = blockIdx.x;          // row block
  const int split = blockIdx.y;
  const int k_begin = split * kspan;
  const int k_end = min(p.K, k_begin + kspan);
  const int n_block = rb * kRowsPerCta;

  if (threadIdx.x < 16) lut[threadIdx.x] = kNF4Levels[threadIdx.x];
  // stage this split's token slice (zero rows >= M and columns >= K)
  for (int i = threadIdx.x; i < kMaxTok * (kspan / 8); i += blockDim.x) {
    const int m = i / (kspan / 8), c = (i % (kspan / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (m < p.M && k_begin + c < k_end)
      v = *reinterpret_cast<const uint4*>(p.x + static_cast<long long>(m) * p.K + k_begin + c);
    *reinterpret_cast<uint4*>(xs + m * xld + c) = v;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  float acc[kRG][4];
#pragma unroll
  for (int i = 0; i < kRG; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  const int n_warp = n_block + warp * kRowsPerWarp;

  // Weights of one 128-wide chunk for the warp's 4 row groups.  Each row
  // group's next chunk is requested right after its current one has been
  // converted, so one chunk of loads stays in flight per row group.
  uint4 raw[kRG][Tr::kLoads];
  float sc[kRG], zc[kRG];
  auto load_rg = [&](int kc, int rg) {
    const int n = n_warp + rg * 8 + g;
    const int k = kc + 32 * q;
    const bool ok = kc < k_end && n < p.N && k < p.K;
    const uint4* src = reinterpret_cast<const uint4*>(
        p.w + static_cast<long long>(ok ? n : 0) * p.row_bytes +
        static_cast<long long>(ok ? k : 0) * Tr::kBitsPerW / 8);
#pragma unroll
    for (int l = 0; l < Tr::kLoads; ++l) raw[rg][l] = ok ? __ldg(src + l) : make_uint4(0, 0, 0, 0);
    sc[rg] = 0.f;
    zc[rg] = 0.f;
    if constexpr (kScheme != 0) {
      if (ok) {
        const long long gi =
            static_cast<long long>(n) * ((p.K + p.group - 1) / p.group) + k / p.group;
        if constexpr (kScheme == kNF4) {
          sc[rg] = __ldg(static_cast<const float*>(p.scales) + gi);
        } else {
          sc[rg] = __half2float(static_cast<const __half*>(p.scales)[gi]);
          zc[rg] = __half2float(p.zeros[gi]);
        }
      }
    }
  };
#pragma unroll
  for (int rg = 0; rg < kRG; ++rg) load_rg(k_begin, rg);
  for (int kc = k_begin; kc < k_end; kc += kChunk) {
    const __nv_bfloat16* x0 = xs + g * xld + (kc - k_begin) + 32 * q;
    const __nv_bfloat16* x8 = x0 + 8 * xld;
#pragma unroll
    for (int rg = 0; rg < kRG; ++rg) {
      uint32_t wbits[16];
      to_bf16_pairs<kScheme>(raw[rg], sc[rg], zc[rg], lut, wbits);
      load_rg(kc + kChunk, rg);  // next chunk of this row group
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        const uint2 lo = *reinterpret_cast<const uint2*>(x0 + 4 * b);
        const uint2 hi = *reinterpret_cast<const uint2*>(x8 + 4 * b);
        const uint32_t af[4] = {lo.x, hi.x, lo.y, hi.y};  // rows g, g+8; slots 2q.., 2q+8..
        mma_bf16_16816(acc[rg], af, wbits[2 * b], wbits[2 * b + 1]);
      }
    }
  }

  // partial tile: rows m = g (c0,c1) and g + 8 (c2,c3); columns n = 2q, 2q+1 of each group
  float* part = p.partials + static_cast<long long>(split) * p.M * p.N;
#pragma unroll
  for (int rg = 0; rg < kRG; ++rg) {
    const int n = n_warp + rg * 8 + 2 * q;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = g + 8 * h;
      if (m < p.M) {
        if (n < p.N) __stcg(part + static_cast<long long>(m) * p.N + n, acc[rg][2 * h]);
        if (n + 1 < p.N) __stcg(part + static_cast<long long>(m) * p.N + n + 1, acc[rg][2 * h + 1]);
      }
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t ticket = atomicAdd(&p.counters[rb], 1u);
    last_flag = ticket == static_cast<uint32_t>(p.splits - 1) ? 1u : 0u;
    if (last_flag) p.counters[rb] = 0;
  }
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  // Final phase (last CTA of this row block).  sT comes from the preceding rank
  // kernel, launched as this grid's programmatic primary: wait for it, then
  // fold its k-slices into shared memory (the token slice is no longer needed).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  float* sts = reinterpret_cast<float*>(smem_g);
  if (p.b != nullptr) {
    for (int i = threadIdx.x; i < p.M * p.r; i += blockDim.x) {
      float t = 0.f;
      for (int s2 = 0; s2 < p.st_splits; ++s2)
        t += __ldcg(p.st + static_cast<long long>(s2) * p.M * p.r + i);
      sts[i] = t;
    }
  }
  __syncthreads();
  const int n = n_block + threadIdx.x;
  if (threadIdx.x >= kRowsPerCta || n >= p.N) return;
  float out[kMaxTok];
#pragma unroll
  for (int m = 0; m < kMaxTok; ++m) {
    out[m] = 0.f;
    if (m < p.M)
      for (int s = 0; s < p.splits; ++s)
        out[m] += __ldcg(p.partials + (static_cast<long long>(s) * p.M + m) * p.N + n);
  }
  if (p.b != nullptr) {
    const __nv_bfloat16* brow = p.b + static_cast<long long>(n) * p.r;
    for (int j0 = 0; j0 < p.r; j0 += 8) {
      const uint4 bv = *reinterpret_cast<const uint4*>(brow + j0);
      const __nv_bfloat162* bp = reinterpret_cast<const __nv_bfloat162*>(&bv);
      float bf[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(bp[i]);
        bf[2 * i] = f.x;
        bf[2 * i + 1] = f.y;
      }
#pragma unroll
      for (int m = 0; m < kMaxTok; ++m) {
        if (m < p.M) {
          const float* sm = sts + m * p.r + j0;
#pragma unroll
          for (int i = 0; i < 8; ++i) out[m] = fmaf(bf[i], sm[i], out[m]);
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < kMaxTok; ++m)
    if (m < p.M) p.y[static_cast<long long>(m) * p.N + n] = __float2bfloat16_rn(out[m]);
}

// Partial sums of sT[m, j] = scale * sum_k x[m, k] A[j, k] for m < M <= 16:
// CTA (j, s) covers the s-th slice of k; thread (m = tid / 16, l = tid % 16)
// walks 8-wide k steps with independent loads, then 16 lanes reduce.  It
// signals its dependent grid (the GEMV) at once so that grid streams weights
// meanwhile; the GEMV adds the slices in order.
__global__ void __launch_bounds__(256) lora_rank_small_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ a, int M, int K, int r,
    int kslice, float scale, float* __restrict__ st) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int j = blockIdx.x, split = blockIdx.y;
  const int m = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int k0 = split * kslice, k1 = min(K, k0 + kslice);
  float acc = 0.f;
  if (m < M) {
    const __nv_bfloat16* ar = a + static_cast<long long>(j) * K;
    const __nv_bfloat16* xr = x + static_cast<long long>(m) * K;
#pragma unroll 4
    for (int k = k0 + l * 8; k < k1; k += 128) {
      const uint4 av = __ldg(reinterpret_cast<const uint4*>(ar + k));
      const uint4 xv = __ldg(reinterpret_cast<const uint4*>(xr + k));
      const __nv_bfloat162* ap = reinterpret_cast<const __nv_bfloat162*>(&av);
      const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 af = __bfloat1622float2(ap[i]), xf = __bfloat1622float2(xp[i]);
        acc = fmaf(xf.x, af.x, acc);
        acc = fmaf(xf.y, af.y, acc);
      }
    }
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (l == 0 && m < M) st[(static_cast<long long>(split) * M + m) * r + j] = acc * scale;
}

template <int kScheme>
int launch_gemv_typed(const GemvArgs& a, cudaStream_t s) {
  GemvParams p;
  p.x = static_cast<const __nv_bfloat16*>(a.x);
  p.w = static_cast<const uint8_t*>(a.w);
  p.scales = a.scales;
  p.zeros = static_cast<const __half*>(a.zeros);
  p.b = static_cast<const __nv_bfloat16*>(a.b);
  p.st = a.st;
  p.st_splits = a.b != nullptr ? rank_small_splits(a.K) : 0;
  p.y = static_cast<__nv_bfloat16*>(a.y);
  p.partials = a.partials;
  p.counters = a.counters;
  p.M = static_cast<int>(a.M);
  p.N = static_cast<int>(a.N);
  p.K = static_cast<int>(a.K);
  p.r = static_cast<int>(a.r);
  p.group = static_cast<int>(a.group);
  p.splits = a.splits;
  p.k_per_split = static_cast<int>(gemv_k_per_split(a.K, a.splits));
  p.row_bytes = a.K * GemvTraits<kScheme>::kBitsPerW / 8;
  p.status = device_status_ptr();
  size_t smem = static_cast<size_t>(kMaxTok) * (p.k_per_split + kXPad) * 2;
  const size_t st_smem = static_cast<size_t>(a.M) * a.r * 4;  // final phase reuses the slice
  if (st_smem > smem) smem = st_smem;
  auto kern = lora_gemv_kernel<kScheme>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) {
      set_error(std::string("gemv attribute: ") + cudaGetErrorString(e));
      return MLORA_ERR_CUDA;
    }
  }
  dim3 grid(static_cast<unsigned>((a.N + kRowsPerCta - 1) / kRowsPerCta),
            static_cast<unsigned>(a.splits));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kGemvWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  LaunchScope scope(kKindGemv, s);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("gemv launch: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

}  // namespace

int64_t gemv_row_blocks(int64_t N) { return (N + kRowsPerCta - 1) / kRowsPerCta; }

int64_t gemv_k_per_split(int64_t K, int splits) {
  const int64_t per = (K + splits - 1) / splits;
  return (per + kChunk - 1) / kChunk * kChunk;
}

int gemv_splits(int64_t N, int64_t K) {
  const int64_t blocks = (N + kRowsPerCta - 1) / kRowsPerCta;
  const int64_t chunks = (K + kChunk - 1) / kChunk;
  int64_t splits = (3 * num_sms()) / blocks;  // one wave at 3 CTAs per SM
  if (splits > chunks) splits = chunks;
  // keep each CTA's staged token slice within 64 KB (16 tokens x bf16)
  while (gemv_k_per_split(K, static_cast<int>(splits)) > 2048) ++splits;
  if (splits < 1) splits = 1;
  return static_cast<int>(splits);
}

int launch_gemv(const GemvArgs& a, cudaStream_t s) {
  if (a.M > kMaxTok) {
    set_error("gemv path takes at most 16 tokens");
    return MLORA_ERR_UNSUPPORTED;
  }
  switch (a.scheme) {
    case 0: return launch_gemv_typed<0>(a, s);
    case kNF4: return launch_gemv_typed<kNF4>(a, s);
    case kINT4: return launch_gemv_typed<kINT4>(a, s);
    case kINT8: return launch_gemv_typed<kINT8>(a, s);
    default: set_error("gemv: unknown scheme"); return MLORA_ERR_INVALID_ARG;
  }
}

int rank_small_splits(int64_t K) {
  const int64_t s = (K + 1023) / 1024;  // ~1024 k per CTA
  return static_cast<int>(s < 1 ? 1 : (s > 16 ? 16 : s));
}

int launch_rank_small(const void* x, const void* a, int64_t M, int64_t K, int64_t r, float scale,
                      float* st, cudaStream_t s) {
  LaunchScope scope(kKindGemv, s);
  const int splits = rank_small_splits(K);
  const int64_t kslice = ((K + splits - 1) / splits + 127) / 128 * 128;
  lora_rank_small_kernel<<<dim3(static_cast<unsigned>(r), static_cast<unsigned>(splits)), 256, 0,
                           s>>>(static_cast<const __nv_bfloat16*>(x),
                                static_cast<const __nv_bfloat16*>(a), static_cast<int>(M),
                                static_cast<int>(K), static_cast<int>(r),
                                static_cast<int>(kslice), scale, st);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("rank_small launch: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

}  // namespace mlora
