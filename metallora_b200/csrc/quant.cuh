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

}  // namespace mlora
