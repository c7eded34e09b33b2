// Quantised base-weight formats of the LoRA path (device side).
//
//   NF4  : codes [N, K/2] bytes (low nibble = even k, high = odd k), absmax
//          [N, ceil(K/bs)] fp32; w = NF4_LEVELS[code] * absmax
//          (kernels/lora_quantized.metal:10-25, :70-74, :122, :135).
//   INT4 : codes [N, K/2] bytes (same nibble order), scale/zero fp16
//          [N, ceil(K/g)]; w = (float(q) - float(zero)) * float(scale)
//          (lora_quantized.metal:17-20, generalised from per-row to per group).
//   INT8 : codes [N, K] bytes, scale/zero as INT4.
// Dequantisation is done in fp32 in exactly the reference's operation order so
// the fp32 values are bit-identical; the tensor-core paths round them to bf16.
#pragma once

#include <stdint.h>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace mlora {

enum QuantScheme : int { kNF4 = 1, kINT4 = 2, kINT8 = 3 };

// The reference's 4-decimal NF4 codebook (lora_quantized.metal:10-15).
__device__ __constant__ static const float kNF4Levels[16] = {
    -1.0f,    -0.6962f, -0.5251f, -0.3949f, -0.2844f, -0.1848f, -0.0911f, 0.0f,
    0.0796f,  0.1609f,  0.2461f,  0.3379f,  0.4407f,  0.5627f,  0.7230f,  1.0f};

__device__ __forceinline__ float dequant_nf4(uint32_t code, float absmax, const float* lut) {
  return __fmul_rn(lut[code], absmax);
}

__device__ __forceinline__ float dequant_int(uint32_t q, float scale, float zero) {
  return __fmul_rn(__fsub_rn(static_cast<float>(q), zero), scale);
}

// Packed fp32 pairs (sm_100 `.f32x2`): low word = first value.  Each half is
// rounded exactly as the scalar __fadd_rn / __fsub_rn / __fmul_rn, so a pair
// routine gives the same bits as two scalar calls.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2_hi(uint64_t v) {
  return __uint_as_float(static_cast<uint32_t>(v >> 32));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// float(q) for the code bytes of `word` selected by `sel0`/`sel1` (byte
// indices 0-3): 2^23 + q is built by a byte permute and 2^23 subtracted,
// which is exact, so the pair equals (float(q0), float(q1)).
__device__ __forceinline__ uint64_t f2_from_bytes(uint32_t word, uint32_t sel0, uint32_t sel1) {
  const uint32_t m0 = __byte_perm(word, 0x4B000000u, 0x7440u | sel0);
  const uint32_t m1 = __byte_perm(word, 0x4B000000u, 0x7440u | sel1);
  const uint64_t magic = (static_cast<uint64_t>(m1) << 32) | m0;
  return f2_add(magic, f2_pack(-8388608.f, -8388608.f));
}

// Pair table of the 4-bit dequantisers: one shared-memory lookup per code
// byte b returns (v(b & 15), v(b >> 4)) -- the two weights of the byte, low
// nibble first -- with v the NF4 level (kNF4) or float(q) (kINT4).  Entry
// (b, c) sits at byte offset 128 b + 8 c, c = thread % 16, so the lanes of a
// half-warp read distinct bank pairs (an LDS.64 of a warp is two wavefronts
// whatever the codes).
constexpr int kPairCopies = 16;

template <int kScheme>
__device__ __forceinline__ void fill_pair_table(uint64_t* t, int tid, int nthreads) {
  for (int i = tid; i < 256 * kPairCopies; i += nthreads) {
    const int b = i / kPairCopies;
    t[i] = kScheme == kNF4 ? f2_pack(kNF4Levels[b & 15], kNF4Levels[b >> 4])
                           : f2_pack(static_cast<float>(b & 15), static_cast<float>(b >> 4));
  }
}

// The four pairs of the 8 nibbles of `w` (byte j -> weights 2j, 2j + 1);
// `tbl_lane` = table base + 8 * (thread % 16).
__device__ __forceinline__ void pair_lookup8(uint32_t w, const char* tbl_lane, uint64_t (&p)[4]) {
  // byte j's offset 128 * byte, taken straight from its bit position
  p[0] = *reinterpret_cast<const uint64_t*>(tbl_lane + ((w << 7) & 0x7F80u));
  p[1] = *reinterpret_cast<const uint64_t*>(tbl_lane + ((w >> 1) & 0x7F80u));
  p[2] = *reinterpret_cast<const uint64_t*>(tbl_lane + ((w >> 9) & 0x7F80u));
  p[3] = *reinterpret_cast<const uint64_t*>(tbl_lane + ((w >> 17) & 0x7F80u));
}

// Eight dequantised weights as packed fp32 pairs, in the scalar order:
// NF4 L[c] * absmax; INT (float(q) - zero) * scale.  w0 holds the eight
// 4-bit codes, or w0/w1 the eight INT8 codes.
template <int kScheme>
__device__ __forceinline__ void dequant8_pairs(uint32_t w0, uint32_t w1, float scale, float zero,
                                               const char* tbl_lane, uint64_t (&p)[4]) {
  if constexpr (kScheme == kINT8) {
    p[0] = f2_from_bytes(w0, 0, 1);
    p[1] = f2_from_bytes(w0, 2, 3);
    p[2] = f2_from_bytes(w1, 0, 1);
    p[3] = f2_from_bytes(w1, 2, 3);
  } else {
    pair_lookup8(w0, tbl_lane, p);
  }
  if constexpr (kScheme != kNF4) {
    const uint64_t zz = f2_pack(zero, zero);
#pragma unroll
    for (int j = 0; j < 4; ++j) p[j] = f2_sub(p[j], zz);
  }
  const uint64_t ss = f2_pack(scale, scale);
#pragma unroll
  for (int j = 0; j < 4; ++j) p[j] = f2_mul(p[j], ss);
}

}  // namespace mlora
