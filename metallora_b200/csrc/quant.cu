// Quantisation, dequantisation and scale re-layout kernels (HBM-bound).
//
// Quantisers (the reference ships none; this project's definition, restated in
// oracle/quant_oracle.py and checked bit-exact against it):
//   NF4 : per (row, block) absmax = max|w|; code = argmin_i |w/absmax - L[i]|
//         (first index on ties); an all-zero block gets absmax 0 and code 7.
//   INT : per (row, group) scale = fp16 round-up of (max - min)/(2^b - 1)
//         (1 when 0), zero = clamp(rint(-min/scale)), q = clamp(rint(w/scale) + zero).
// Dequantisers follow the reference shaders' fp32 arithmetic
// (kernels/lora_quantized.metal:17-25).
#include <algorithm>
#include <atomic>
#include <string>

#include "internal.h"
#include "quant.cuh"
#include "../../include/metallora_b200.h"

namespace mlora {
namespace {

template <typename T>
__device__ __forceinline__ float to_f32(T v) {
  return static_cast<float>(v);
}

// One warp per (row, block); lanes stride over the block's elements.
template <typename T>
__global__ void quantize_nf4_kernel(const T* __restrict__ w, int64_t N, int64_t K, int64_t bs,
                                    uint8_t* __restrict__ codes, float* __restrict__ absmax) {
  const int64_t nblk = (K + bs - 1) / bs;
  const int64_t warp_global = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_global >= N * nblk) return;
  const int64_t row = warp_global / nblk, blk = warp_global % nblk;
  const int64_t k0 = blk * bs, k1 = min(K, k0 + bs);
  const T* wr = w + row * K;
  float am = 0.f;
  for (int64_t k = k0 + lane; k < k1; k += 32) am = fmaxf(am, fabsf(to_f32(wr[k])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  if (lane == 0) absmax[row * nblk + blk] = am;
  const float safe = am == 0.f ? 1.f : am;
  // each lane produces whole bytes (k even, k+1)
  for (int64_t k = k0 + 2 * lane; k < k1; k += 64) {
    uint32_t byte = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t code = 7;
      if (am != 0.f && k + h < K) {
        const float v = __fdiv_rn(to_f32(wr[k + h]), safe);
        float best = fabsf(__fsub_rn(v, kNF4Levels[0]));
        code = 0;
#pragma unroll
        for (int i = 1; i < 16; ++i) {
          const float d = fabsf(__fsub_rn(v, kNF4Levels[i]));
          if (d < best) best = d, code = i;
        }
      }
      byte |= code << (4 * h);
    }
    codes[row * (K / 2) + k / 2] = static_cast<uint8_t>(byte);
  }
}

template <typename T, int kBits>
__global__ void quantize_int_kernel(const T* __restrict__ w, int64_t N, int64_t K, int64_t g,
                                    uint8_t* __restrict__ codes, __half* __restrict__ scales,
                                    __half* __restrict__ zeros) {
  const int64_t ng = (K + g - 1) / g;
  const int64_t warp_global = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_global >= N * ng) return;
  const int64_t row = warp_global / ng, grp = warp_global % ng;
  const int64_t k0 = grp * g, k1 = min(K, k0 + g);
  const T* wr = w + row * K;
  float mn = INFINITY, mx = -INFINITY;
  for (int64_t k = k0 + lane; k < k1; k += 32) {
    const float v = to_f32(wr[k]);
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const float qmax = static_cast<float>((1 << kBits) - 1);
  __half sh = __float2half_ru(__fdiv_rn(__fsub_rn(mx, mn), qmax));
  if (__half2float(sh) == 0.f) sh = __float2half(1.f);
  const float s = __half2float(sh);
  const float zero = fminf(fmaxf(rintf(__fdiv_rn(-mn, s)), 0.f), qmax);
  if (lane == 0) {
    scales[row * ng + grp] = sh;
    zeros[row * ng + grp] = __float2half(zero);
  }
  if (kBits == 8) {
    for (int64_t k = k0 + lane; k < k1; k += 32) {
      const float q = fminf(fmaxf(__fadd_rn(rintf(__fdiv_rn(to_f32(wr[k]), s)), zero), 0.f), qmax);
      codes[row * K + k] = static_cast<uint8_t>(q);
    }
  } else {
    for (int64_t k = k0 + 2 * lane; k < k1; k += 64) {
      uint32_t byte = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (k + h < K) {
          const float q =
              fminf(fmaxf(__fadd_rn(rintf(__fdiv_rn(to_f32(wr[k + h]), s)), zero), 0.f), qmax);
          byte |= static_cast<uint32_t>(q) << (4 * h);
        }
      }
      codes[row * (K / 2) + k / 2] = static_cast<uint8_t>(byte);
    }
  }
}

template <typename O>
__device__ __forceinline__ O from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

template <typename O>
__global__ void dequantize_kernel(int scheme, const uint8_t* __restrict__ codes,
                                  const void* __restrict__ scales, const __half* __restrict__ zeros,
                                  int64_t N, int64_t K, int64_t g, O* __restrict__ out) {
  __shared__ float lut[16];
  if (threadIdx.x < 16) lut[threadIdx.x] = kNF4Levels[threadIdx.x];
  __syncthreads();
  const int64_t total = N * K;
  const int64_t ng = (K + g - 1) / g;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / K, k = i % K;
    float v;
    if (scheme == kINT8) {
      const float s = __half2float(static_cast<const __half*>(scales)[row * ng + k / g]);
      const float z = __half2float(zeros[row * ng + k / g]);
      v = dequant_int(codes[row * K + k], s, z);
    } else {
      const uint32_t byte = codes[row * (K / 2) + k / 2];
      const uint32_t q = (k & 1) ? (byte >> 4) & 0xF : byte & 0xF;
      if (scheme == kNF4) {
        v = dequant_nf4(q, static_cast<const float*>(scales)[row * ng + k / g], lut);
      } else {
        const float s = __half2float(static_cast<const __half*>(scales)[row * ng + k / g]);
        const float z = __half2float(zeros[row * ng + k / g]);
        v = dequant_int(q, s, z);
      }
    }
    out[i] = from_f32<O>(v);
  }
}

// Vectorised dequantiser for K % 8 == 0 and group % 8 == 0: one item = 8
// consecutive weights of one row (4 code bytes for 4-bit, 8 for INT8), so item
// i reads codes at byte i*4 (i*8) and writes out[i*8 .. i*8+7] -- every warp
// load and store is one contiguous run.  Each thread keeps kUnroll items'
// loads in flight.
//
// The arithmetic is the scalar kernel's, done on packed fp32 pairs (each half
// rounds as the scalar op, so the outputs are identical):
//   * 4-bit: one shared-memory lookup per code byte returns the pair
//     (v(low nibble), v(high nibble)), v = the NF4 level or float(q); the
//     table is replicated so each lane of a half-warp reads its own bank pair;
//   * INT8: float(q) = (2^23 + q) - 2^23, the first built by a byte permute;
//   * then (INT) - zero, * scale, and a packed round to bf16 / fp16.
// When the groups tile the rows (K % group == 0) and group/8 is a power of
// two, an item's scale index is item >> shift (no division).
constexpr int kDqVecThreads = 512;

template <typename O>
__device__ __forceinline__ void store8(O* dst, const uint64_t (&p)[4]) {
  if constexpr (sizeof(O) == 4) {
    reinterpret_cast<float4*>(dst)[0] = make_float4(f2_lo(p[0]), f2_hi(p[0]), f2_lo(p[1]), f2_hi(p[1]));
    reinterpret_cast<float4*>(dst)[1] = make_float4(f2_lo(p[2]), f2_hi(p[2]), f2_lo(p[3]), f2_hi(p[3]));
  } else {
    uint4 u;  // round-to-nearest-even, as from_f32
    u.x = pack2<O>(f2_lo(p[0]), f2_hi(p[0]));
    u.y = pack2<O>(f2_lo(p[1]), f2_hi(p[1]));
    u.z = pack2<O>(f2_lo(p[2]), f2_hi(p[2]));
    u.w = pack2<O>(f2_lo(p[3]), f2_hi(p[3]));
    *reinterpret_cast<uint4*>(dst) = u;
  }
}

template <int kScheme, typename O, typename Idx, bool kShift>
__global__ void __launch_bounds__(kDqVecThreads) dequantize_vec_kernel(
    const uint8_t* __restrict__ codes, const void* __restrict__ scales,
    const __half* __restrict__ zeros, Idx items, Idx items_per_row, Idx ng, Idx g8,
    int g8_shift, O* __restrict__ out) {
  constexpr int kUnroll = 4;
  constexpr bool kTable = kScheme != kINT8;
  __shared__ uint64_t table[kTable ? 256 * kPairCopies : 1];
  if constexpr (kTable) {
    fill_pair_table<kScheme>(table, threadIdx.x, blockDim.x);
    __syncthreads();
  }
  const char* tbl_lane = reinterpret_cast<const char*>(table) + (threadIdx.x % kPairCopies) * 8;
  const Idx stride = static_cast<Idx>(gridDim.x) * blockDim.x;
  for (Idx base = static_cast<Idx>(blockIdx.x) * blockDim.x + threadIdx.x; base < items;
       base += stride * kUnroll) {
    uint2 raw[kUnroll];
    float s[kUnroll], z[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const Idx it = base + u * stride;
      raw[u] = make_uint2(0, 0);
      s[u] = 0.f;
      z[u] = 0.f;
      if (it < items) {
        Idx gi;
        if constexpr (kShift) {
          gi = it >> g8_shift;
        } else {
          const Idx row = it / items_per_row;
          gi = row * ng + (it - row * items_per_row) / g8;
        }
        if constexpr (kScheme == kINT8) {
          raw[u] = __ldg(reinterpret_cast<const uint2*>(codes) + it);
        } else {
          raw[u].x = __ldg(reinterpret_cast<const uint32_t*>(codes) + it);
        }
        if constexpr (kScheme == kNF4) {
          s[u] = __ldg(static_cast<const float*>(scales) + gi);
        } else {
          s[u] = __half2float(static_cast<const __half*>(scales)[gi]);
          z[u] = __half2float(zeros[gi]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const Idx it = base + u * stride;
      if (it >= items) break;
      uint64_t p[4];
      dequant8_pairs<kScheme>(raw[u].x, raw[u].y, s[u], z[u], tbl_lane, p);
      store8<O>(out + it * 8, p);
    }
  }
}

// src [rows, cols] -> dst [cols, ld] (ld >= rows) for 4-byte elements;
// columns rows..ld-1 of dst are zeroed.
__global__ void transpose_f32_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                                     int64_t ld, float* __restrict__ dst) {
  __shared__ float tile[32][33];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32, c0 = static_cast<int64_t>(blockIdx.x) * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (r < rows && c < cols) ? src[r * cols + c] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (c < cols && r < ld) dst[c * ld + r] = tile[threadIdx.x][i];
  }
}

// scale/zero fp16 [rows, cols] -> interleaved (scale, zero) pairs [cols, rows].
__global__ void pack_scale_zero_kernel(const __half* __restrict__ s, const __half* __restrict__ z,
                                       int64_t rows, int64_t cols, int64_t ld,
                                       __half2* __restrict__ dst) {
  __shared__ __half2 tile[32][33];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32, c0 = static_cast<int64_t>(blockIdx.x) * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (r < rows && c < cols) ? __halves2half2(s[r * cols + c], z[r * cols + c])
                                                  : __halves2half2(__float2half(0.f), __float2half(0.f));
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (c < cols && r < ld) dst[c * ld + r] = tile[threadIdx.x][i];
  }
}

int grid_1d(int64_t items, int per_block) {
  int64_t g = (items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 32;
  if (g > cap) g = cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

int launched(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

}  // namespace

int launch_quantize(const void* w, int w_dtype, int64_t N, int64_t K, int scheme, int64_t g,
                    void* codes, void* scales, void* zeros, cudaStream_t s) {
  LaunchScope scope(kKindQuant, s);
  const int64_t groups = N * ((K + g - 1) / g);
  const int threads = 256;
  const int64_t blocks64 = (groups * 32 + threads - 1) / threads;
  if (blocks64 > (int64_t(1) << 31) - 1) {
    set_error("quantize: too many groups");
    return MLORA_ERR_UNSUPPORTED;
  }
  const unsigned blocks = static_cast<unsigned>(blocks64);
  auto* c8 = static_cast<uint8_t*>(codes);
#define MLORA_Q_DISPATCH(T)                                                                      \
  do {                                                                                           \
    const T* wt = static_cast<const T*>(w);                                                      \
    if (scheme == kNF4)                                                                          \
      quantize_nf4_kernel<T><<<blocks, threads, 0, s>>>(wt, N, K, g, c8, static_cast<float*>(scales)); \
    else if (scheme == kINT4)                                                                    \
      quantize_int_kernel<T, 4><<<blocks, threads, 0, s>>>(wt, N, K, g, c8,                      \
          static_cast<__half*>(scales), static_cast<__half*>(zeros));                            \
    else                                                                                         \
      quantize_int_kernel<T, 8><<<blocks, threads, 0, s>>>(wt, N, K, g, c8,                      \
          static_cast<__half*>(scales), static_cast<__half*>(zeros));                            \
  } while (0)
  if (w_dtype == MLORA_DTYPE_F32)
    MLORA_Q_DISPATCH(float);
  else if (w_dtype == MLORA_DTYPE_BF16)
    MLORA_Q_DISPATCH(__nv_bfloat16);
  else
    MLORA_Q_DISPATCH(__half);
#undef MLORA_Q_DISPATCH
  return launched("quantize");
}

namespace {
template <int kScheme, typename O, typename Idx>
void launch_dequantize_vec(const uint8_t* codes, const void* scales, const __half* zeros,
                           int64_t N, int64_t K, int64_t g, O* out, cudaStream_t s) {
  const int64_t items = N * K / 8;
  const int64_t g8 = g / 8;
  int shift = 0;
  while ((int64_t(1) << shift) < g8) ++shift;
  const bool fast = K % g == 0 && (int64_t(1) << shift) == g8;
  auto* kernel = fast ? dequantize_vec_kernel<kScheme, O, Idx, true>
                      : dequantize_vec_kernel<kScheme, O, Idx, false>;
  // persistent-style: one wave of resident blocks, each filling its table once
  static std::atomic<int> per_sm[2] = {{0}, {0}};
  int occ = per_sm[fast ? 1 : 0].load(std::memory_order_relaxed);
  if (occ == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kDqVecThreads, 0) !=
        cudaSuccess) {
      occ = 1;
      (void)cudaGetLastError();  // the launch check below must see the launch's own status
    }
    occ = std::max(occ, 1);
    per_sm[fast ? 1 : 0].store(occ, std::memory_order_relaxed);
  }
  int64_t grid = (items + int64_t(4) * kDqVecThreads - 1) / (int64_t(4) * kDqVecThreads);
  grid = std::max<int64_t>(1, std::min<int64_t>(grid, int64_t(occ) * num_sms()));
  kernel<<<static_cast<int>(grid), kDqVecThreads, 0, s>>>(
      codes, scales, zeros, static_cast<Idx>(items), static_cast<Idx>(K / 8),
      static_cast<Idx>((K + g - 1) / g), static_cast<Idx>(g8), shift, out);
}

template <typename O>
void dispatch_dequantize_vec(int scheme, const uint8_t* codes, const void* scales,
                             const __half* zeros, int64_t N, int64_t K, int64_t g, O* out,
                             cudaStream_t s) {
  // 32-bit index arithmetic whenever the item count and the scale index fit
  const bool small = N * K / 8 < (int64_t(1) << 31) && N * ((K + g - 1) / g) < (int64_t(1) << 31);
#define MLORA_DQ(SCH)                                                                            \
  (small ? launch_dequantize_vec<SCH, O, uint32_t>(codes, scales, zeros, N, K, g, out, s)         \
         : launch_dequantize_vec<SCH, O, int64_t>(codes, scales, zeros, N, K, g, out, s))
  if (scheme == kNF4)
    MLORA_DQ(kNF4);
  else if (scheme == kINT4)
    MLORA_DQ(kINT4);
  else
    MLORA_DQ(kINT8);
#undef MLORA_DQ
}
}  // namespace

int launch_dequantize(int scheme, const void* codes, const void* scales, const void* zeros,
                      int64_t N, int64_t K, int64_t g, void* out, int out_dtype, cudaStream_t s) {
  LaunchScope scope(kKindQuant, s);
  const auto* c8 = static_cast<const uint8_t*>(codes);
  const auto* z = static_cast<const __half*>(zeros);
  const auto addr = [](const void* p) { return reinterpret_cast<uintptr_t>(p); };
  const bool vec = K % 8 == 0 && g % 8 == 0 && addr(out) % 16 == 0 &&
                   addr(codes) % (scheme == kINT8 ? 8 : 4) == 0 && addr(scales) % 4 == 0;
  if (vec) {
    if (out_dtype == MLORA_DTYPE_F32)
      dispatch_dequantize_vec(scheme, c8, scales, z, N, K, g, static_cast<float*>(out), s);
    else if (out_dtype == MLORA_DTYPE_BF16)
      dispatch_dequantize_vec(scheme, c8, scales, z, N, K, g, static_cast<__nv_bfloat16*>(out), s);
    else
      dispatch_dequantize_vec(scheme, c8, scales, z, N, K, g, static_cast<__half*>(out), s);
    return launched("dequantize");
  }
  const int grid = grid_1d(N * K, 256);
  if (out_dtype == MLORA_DTYPE_F32)
    dequantize_kernel<float><<<grid, 256, 0, s>>>(scheme, c8, scales, z, N, K, g,
                                                   static_cast<float*>(out));
  else if (out_dtype == MLORA_DTYPE_BF16)
    dequantize_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(scheme, c8, scales, z, N, K, g,
                                                           static_cast<__nv_bfloat16*>(out));
  else
    dequantize_kernel<__half><<<grid, 256, 0, s>>>(scheme, c8, scales, z, N, K, g,
                                                   static_cast<__half*>(out));
  return launched("dequantize");
}

int launch_transpose_f32(const float* src, int64_t rows, int64_t cols, int64_t ld, float* dst,
                         cudaStream_t s) {
  LaunchScope scope(kKindElementwise, s);
  dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((ld + 31) / 32));
  transpose_f32_kernel<<<grid, dim3(32, 8), 0, s>>>(src, rows, cols, ld, dst);
  return launched("transpose_f32");
}

int launch_pack_scale_zero(const void* scales, const void* zeros, int64_t rows, int64_t cols,
                           int64_t ld, void* dst, cudaStream_t s) {
  LaunchScope scope(kKindElementwise, s);
  dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((ld + 31) / 32));
  pack_scale_zero_kernel<<<grid, dim3(32, 8), 0, s>>>(static_cast<const __half*>(scales),
                                                     static_cast<const __half*>(zeros), rows,
                                                     cols, ld, static_cast<__half2*>(dst));
  return launched("pack_scale_zero");
}

}  // namespace mlora
