// Persistent tcgen05 GEMM over a quantised base weight, dequantised inside the
// main loop:
//
//     D[M, N] = X[M, K] . deq(Wq)^T  +  X2[M, R] . W2^T
//
//   forward  y  = x . deq(W0)^T + (s x A^T) . B^T          (K-major W tiles)
//   backward dx = dy . deq(W0)  + (s dy B) . A              (MN-major W tiles)
// replacing qlora_forward_nf4 / qlora_forward_int4 (kernels/lora_quantized.metal:29-164),
// which re-read and re-dequantised every weight for every token.
//
// One-CTA kernel (M < 256; the CTA-pair variant below takes M >= 256).
// Warp roles (14 warps, one CTA per SM):
//   warp 0      TMA producer: bf16 X tiles [128 x 64] into a 4-stage ring, and the
//               packed codes + per-block scales of the matching W tile into a
//               4-stage "raw" ring (plain, unswizzled boxes).
//   warp 1      TMEM owner and UMMA issuer (M 128, N 256, K 16; accumulators
//               double-buffered in TMEM).
//   warps 2-5   epilogue (as in the dense kernel).
//   warps 6-13  dequantisers: each thread turns one 64-element row of the raw
//               tile into bf16 -- value = bf16_rn(fp32 dequant), the reference's
//               fp32 arithmetic (4-bit rows through a per-row register
//               codebook) -- and stores it 16 bytes at a time into the
//               128-byte-swizzled layout UMMA reads (2-stage ring).  For the
//               rank block they copy B (forward) or A (backward) rows instead.
// Every wait is bounded (see ptx.cuh).
#include <algorithm>
#include <cstdlib>
#include <string>

#include "internal.h"
#include "ptx.cuh"
#include "quant.cuh"
#include "../../include/metallora_b200.h"

namespace mlora {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStagesX = 4;
constexpr int kStagesR = 4;
constexpr int kStagesW = 2;
constexpr uint32_t kXTileBytes = kBM * kBK * 2;
constexpr uint32_t kWTileBytes = kBN * kBK * 2;
constexpr uint32_t kMNBoxBytes = 64 * kBK * 2;
constexpr int kEpiWarps = 4;
constexpr int kDqWarps = 8;
constexpr int kDqThreads = 32 * kDqWarps;
constexpr int kThreads = 64 + 32 * kEpiWarps + kDqThreads;
constexpr uint32_t kTmemCols = 512;

template <int kScheme>
struct QTraits {
  static constexpr int kBits = kScheme == kINT8 ? 8 : 4;
  static constexpr uint32_t kCodeBytes = kBN * kBK * kBits / 8;  // 8 or 16 KB per tile
  static constexpr uint32_t kScaleBytes = 1024;                   // room for any scale box
  static constexpr uint32_t kRawBytes = kCodeBytes + kScaleBytes;
};

template <int kScheme>
constexpr size_t smem_bytes() {
  return 1024 + kStagesX * kXTileBytes + kStagesW * kWTileBytes +
         kStagesR * QTraits<kScheme>::kRawBytes + 512;
}

struct QGemmParams {
  int M, N;
  int num_kb_main, num_kb_extra, R;
  int tiles_n, num_tiles;
  int group;             // scale block along the weight's in-feature axis
  uint32_t scale_box_bytes;
  void* d;
  long long ldd;
  const __nv_bfloat16* up;  // forward: B [N, r]; backward: A [r, K]
  int up_rows;             // r
  long long up_ld;         // row stride of `up`
  long long up_cols;       // forward: r ; backward: K (valid columns)
  uint32_t* status;
};

// Stores 8 bf16 values (one 16-byte chunk) into a 128-byte swizzled row.
__device__ __forceinline__ void st_chunk(uint8_t* row_base, uint32_t row, uint32_t chunk,
                                         uint4 v) {
  *reinterpret_cast<uint4*>(row_base + ((chunk ^ (row & 7u)) << 4)) = v;
}

// Dequantises 8 consecutive INT8 weights held in w0/w1 into a 16-byte chunk
// of bf16 (packed fp32 pairs, the scalar rounding).
__device__ __forceinline__ uint4 dq8_int8(uint32_t w0, uint32_t w1, float scale, float zero) {
  uint64_t p[4];
  dequant8_pairs<kINT8>(w0, w1, scale, zero, nullptr, p);
  return make_uint4(pack2<__nv_bfloat16>(f2_lo(p[0]), f2_hi(p[0])),
                    pack2<__nv_bfloat16>(f2_lo(p[1]), f2_hi(p[1])),
                    pack2<__nv_bfloat16>(f2_lo(p[2]), f2_hi(p[2])),
                    pack2<__nv_bfloat16>(f2_lo(p[3]), f2_hi(p[3])));
}

// A 4-bit row of 64 weights shares one scale (and zero): its codes take at
// most 16 values v(c) = bf16((L[c] or float(c) - zero) * scale), computed here
// once in the scalar rounding and kept as byte planes: lo[t] holds the low
// bytes of v(4t .. 4t+3), hi[t] their high bytes.
template <int kScheme>
__device__ __forceinline__ void row_codebook(float s, float z, uint32_t (&lo)[4],
                                             uint32_t (&hi)[4]) {
  const uint64_t ss = f2_pack(s, s), zz = f2_pack(z, z);
  uint32_t v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint64_t p;
    if constexpr (kScheme == kNF4)
      p = f2_pack(kNF4Levels[2 * j], kNF4Levels[2 * j + 1]);
    else
      p = f2_sub(f2_pack(static_cast<float>(2 * j), static_cast<float>(2 * j + 1)), zz);
    p = f2_mul(p, ss);
    v[j] = pack2<__nv_bfloat16>(f2_lo(p), f2_hi(p));
  }
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    lo[t] = __byte_perm(v[2 * t], v[2 * t + 1], 0x6420);
    hi[t] = __byte_perm(v[2 * t], v[2 * t + 1], 0x7531);
  }
}

// Eight bf16 weights (one word of 4-bit codes, nibble i = weight i) from the
// row's codebook, by byte permutes only: for four codes at a time, one permute
// per plane picks the byte of v(c & 7) from each 8-entry half, a second keeps
// the half that bit 3 of the code names, a third interleaves low and high
// bytes into bf16 pairs.
__device__ __forceinline__ uint4 codebook8(uint32_t w, const uint32_t (&lo)[4],
                                           const uint32_t (&hi)[4]) {
  uint32_t out[4];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t c = h ? (w >> 16) : w;        // a permute reads selector bits 0-15
    const uint32_t sel = c & 0x7777u;             // c & 7 per nibble
    const uint32_t msel = ((c >> 1) & 0x4444u) | 0x3210u;  // byte i, or byte i of the upper half
    const uint32_t l = __byte_perm(__byte_perm(lo[0], lo[1], sel), __byte_perm(lo[2], lo[3], sel), msel);
    const uint32_t u = __byte_perm(__byte_perm(hi[0], hi[1], sel), __byte_perm(hi[2], hi[3], sel), msel);
    out[2 * h] = __byte_perm(l, u, 0x5140);       // weights 4h, 4h + 1
    out[2 * h + 1] = __byte_perm(l, u, 0x7362);   // weights 4h + 2, 4h + 3
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

template <int kScheme>
__device__ __forceinline__ void scale_zero(const uint8_t* scales, uint32_t idx, float& s,
                                           float& z) {
  if constexpr (kScheme == kNF4) {
    s = reinterpret_cast<const float*>(scales)[idx];
    z = 0.f;
  } else {
    const __half2 sz = reinterpret_cast<const __half2*>(scales)[idx];
    s = __low2float(sz);
    z = __high2float(sz);
  }
}

// One thread converts one 64-element weight row of the raw tile.
template <int kScheme>
__device__ __forceinline__ void dequant_row(const uint8_t* codes, float s, float z,
                                            uint8_t* out_row, uint32_t swz_row) {
  if constexpr (kScheme == kINT8) {
    const uint4* c = reinterpret_cast<const uint4*>(codes);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 u = c[q];
      st_chunk(out_row, swz_row, 2 * q, dq8_int8(u.x, u.y, s, z));
      st_chunk(out_row, swz_row, 2 * q + 1, dq8_int8(u.z, u.w, s, z));
    }
  } else {
    uint32_t lo[4], hi[4];
    row_codebook<kScheme>(s, z, lo, hi);
    const uint4* c = reinterpret_cast<const uint4*>(codes);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint4 u = c[q];
      st_chunk(out_row, swz_row, 4 * q + 0, codebook8(u.x, lo, hi));
      st_chunk(out_row, swz_row, 4 * q + 1, codebook8(u.y, lo, hi));
      st_chunk(out_row, swz_row, 4 * q + 2, codebook8(u.z, lo, hi));
      st_chunk(out_row, swz_row, 4 * q + 3, codebook8(u.w, lo, hi));
    }
  }
}

template <int kScheme, bool kWMN>
__global__ void __launch_bounds__(kThreads, 1)
    qlora_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_x2,
                      const __grid_constant__ CUtensorMap tm_codes,
                      const __grid_constant__ CUtensorMap tm_scales, const QGemmParams p) {
  using Tr = QTraits<kScheme>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint8_t* xs = smem;
  uint8_t* ws = xs + kStagesX * kXTileBytes;
  uint8_t* rs = ws + kStagesW * kWTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(rs + kStagesR * Tr::kRawBytes);
  uint64_t* x_full = bars;
  uint64_t* x_empty = x_full + kStagesX;
  uint64_t* r_full = x_empty + kStagesX;
  uint64_t* r_empty = r_full + kStagesR;
  uint64_t* w_full = r_empty + kStagesR;
  uint64_t* w_empty = w_full + kStagesW;
  uint64_t* acc_full = w_empty + kStagesW;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesX; ++s) mbar_init(&x_full[s], 1), mbar_init(&x_empty[s], 1);
    for (int s = 0; s < kStagesR; ++s) mbar_init(&r_full[s], 1), mbar_init(&r_empty[s], 1);
    for (int s = 0; s < kStagesW; ++s) mbar_init(&w_full[s], 1), mbar_init(&w_empty[s], 1);
    for (int b = 0; b < 2; ++b) mbar_init(&acc_full[b], 1), mbar_init(&acc_empty[b], kEpiWarps * 32);
    mbar_init(drain_bar, 1);
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_codes);
    prefetch_tmap(&tm_scales);
    if (p.num_kb_extra > 0) prefetch_tmap(&tm_x2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_kb = p.num_kb_main + p.num_kb_extra;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (elect_one()) {
      uint32_t sx = 0, px = 0, sr = 0, pr = 0;
      bool armed_x[kStagesX], armed_r[kStagesR];
      uint32_t par_x[kStagesX], par_r[kStagesR];
      for (int s = 0; s < kStagesX; ++s) armed_x[s] = false, par_x[s] = 0;
      for (int s = 0; s < kStagesR; ++s) armed_r[s] = false, par_r[s] = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / p.tiles_n) * kBM;
        const int n0 = (tile % p.tiles_n) * kBN;
        for (int kb = 0; kb < total_kb && ok; ++kb) {
          const bool extra = kb >= p.num_kb_main;
          if (!mbar_wait(&x_empty[sx], px ^ 1u, p.status, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&x_full[sx], kXTileBytes);
          armed_x[sx] = true;
          par_x[sx] = px;
          if (extra)
            tma_load_2d(xs + sx * kXTileBytes, &tm_x2, &x_full[sx], (kb - p.num_kb_main) * kBK, m0);
          else
            tma_load_2d(xs + sx * kXTileBytes, &tm_x, &x_full[sx], kb * kBK, m0);
          if (++sx == kStagesX) sx = 0, px ^= 1u;
          if (extra) continue;
          if (!mbar_wait(&r_empty[sr], pr ^ 1u, p.status, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* raw = rs + sr * Tr::kRawBytes;
          mbar_arrive_expect_tx(&r_full[sr], Tr::kCodeBytes + p.scale_box_bytes);
          armed_r[sr] = true;
          par_r[sr] = pr;
          if constexpr (kWMN) {
            // rows: the reduction index n in [kb*64, kb*64+64); bytes of out-features n0..n0+255
            tma_load_2d(raw, &tm_codes, &r_full[sr], n0 * Tr::kBits / 8, kb * kBK);
            tma_load_2d(raw + Tr::kCodeBytes, &tm_scales, &r_full[sr], kb * kBK,
                        n0 / p.group);
          } else {
            tma_load_2d(raw, &tm_codes, &r_full[sr], kb * kBK * Tr::kBits / 8, n0);
            tma_load_2d(raw + Tr::kCodeBytes, &tm_scales, &r_full[sr], n0,
                        (kb * kBK) / p.group);
          }
          if (++sr == kStagesR) sr = 0, pr ^= 1u;
        }
      }
      for (int s = 0; s < kStagesX; ++s)
        if (armed_x[s]) mbar_wait(&x_full[s], par_x[s], p.status, kDevTimeoutDrain);
      for (int s = 0; s < kStagesR; ++s)
        if (armed_r[s]) mbar_wait(&r_full[s], par_r[s], p.status, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA --
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_f16(kBM, kBN, false, kWMN, true);
      uint32_t sx = 0, px = 0, sw = 0, pw = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++local) {
        const uint32_t buf = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1) & 1u;
        if (!mbar_wait(&acc_empty[buf], use ^ 1u, p.status, kDevTimeoutAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * kBN;
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&x_full[sx], px, p.status, kDevTimeoutFull) ||
              !mbar_wait(&w_full[sw], pw, p.status, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sxa = smem_u32(xs + sx * kXTileBytes);
          const uint32_t swa = smem_u32(ws + sw * kWTileBytes);
          int nk = 4;
          if (kb >= p.num_kb_main) {
            const int rem = p.R - (kb - p.num_kb_main) * kBK;
            nk = rem >= kBK ? 4 : rem / 16;
          }
          for (int k = 0; k < nk; ++k) {
            uint64_t bd;
            if constexpr (kWMN)
              bd = desc_mnmajor_sw128(swa, k, kMNBoxBytes);
            else
              bd = desc_kmajor_sw128(swa, k);
            umma_f16(d_tmem, desc_kmajor_sw128(sxa, k), bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&x_empty[sx]);
          umma_commit(&w_empty[sw]);
          if (++sx == kStagesX) sx = 0, px ^= 1u;
          if (++sw == kStagesW) sw = 0, pw ^= 1u;
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
      }
      umma_commit(drain_bar);
      mbar_wait(drain_bar, 0, p.status, kDevTimeoutDrain);
    }
  } else if (warp < 2 + kEpiWarps) {
    // ----------------------------------------------------------- epilogue --
    const uint32_t quarter = warp & 3u;
    const uint32_t row = quarter * 32 + lane;
    const int vec = (p.N % 8 == 0 && p.ldd % 8 == 0) ? 1 : 0;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      const uint32_t buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1) & 1u;
      if (!mbar_wait(&acc_full[buf], use, p.status, kDevTimeoutAccFull)) break;
      tc_fence_after();
      const int m = (tile / p.tiles_n) * kBM + static_cast<int>(row);
      const int n_base = (tile % p.tiles_n) * kBN;
      __nv_bfloat16* out_row =
          reinterpret_cast<__nv_bfloat16*>(p.d) + static_cast<long long>(m) * p.ldd + n_base;
      const uint32_t taddr = tmem_base + ((quarter * 32u) << 16) + buf * kBN;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + c * 32, r);
        tmem_ld_wait();
        if (m < p.M) {
          const int n0 = n_base + c * 32;
          if (!vec) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (n0 + i < p.N) out_row[c * 32 + i] = __float2bfloat16_rn(__uint_as_float(r[i]));
            continue;
          }
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = pack2<__nv_bfloat16>(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (n0 + q * 8 < p.N)
              *reinterpret_cast<uint4*>(out_row + c * 32 + q * 8) =
                  make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  } else {
    // -------------------------------------------------------- dequantisers --
    const uint32_t t = threadIdx.x - (64 + 32 * kEpiWarps);  // 0..255
    uint32_t sr = 0, pr = 0, sw = 0, pw = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      const int n0 = (tile % p.tiles_n) * kBN;
      for (int kb = 0; kb < total_kb; ++kb) {
        const bool extra = kb >= p.num_kb_main;
        if (!mbar_wait(&w_empty[sw], pw ^ 1u, p.status, kDevTimeoutEmpty)) {
          ok = false;
          break;
        }
        uint8_t* wtile = ws + sw * kWTileBytes;
        if (!extra) {
          if (!mbar_wait(&r_full[sr], pr, p.status, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          const uint8_t* raw = rs + sr * Tr::kRawBytes;
          const uint8_t* scales = raw + Tr::kCodeBytes;
          float s, z;
          if constexpr (kWMN) {
            const uint32_t row = t & 63u, box = t >> 6;
            const uint32_t srow = (box * 64u) / static_cast<uint32_t>(p.group);
            scale_zero<kScheme>(scales, srow * 64u + row, s, z);
            dequant_row<kScheme>(raw + row * (kBN * Tr::kBits / 8) + box * (64 * Tr::kBits / 8),
                                 s, z, wtile + box * kMNBoxBytes + row * 128u, row);
          } else {
            scale_zero<kScheme>(scales, t, s, z);
            dequant_row<kScheme>(raw + t * (kBK * Tr::kBits / 8), s, z, wtile + t * 128u, t);
          }
        } else {
          // rank block: copy 64 columns of the up-projection operand (zero padded)
          const int j0 = (kb - p.num_kb_main) * kBK;
          if constexpr (kWMN) {
            const uint32_t row = t & 63u, box = t >> 6;
            const int j = j0 + static_cast<int>(row);
            uint8_t* out_row = wtile + box * kMNBoxBytes + row * 128u;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const long long col = n0 + box * 64 + c * 8;
              uint4 v = make_uint4(0, 0, 0, 0);
              if (j < p.up_rows && col < p.up_cols)
                v = *reinterpret_cast<const uint4*>(p.up + static_cast<long long>(j) * p.up_ld + col);
              st_chunk(out_row, row, c, v);
            }
          } else {
            const long long n = n0 + static_cast<long long>(t);
            uint8_t* out_row = wtile + t * 128u;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const int j = j0 + c * 8;
              uint4 v = make_uint4(0, 0, 0, 0);
              if (n < p.N && j < p.up_rows)
                v = *reinterpret_cast<const uint4*>(p.up + n * p.up_ld + j);
              st_chunk(out_row, t, c, v);
            }
          }
        }
        fence_proxy_async_smem();
        named_bar_sync(2, kDqThreads);
        if (t == 0) {
          mbar_arrive(&w_full[sw]);
          if (!extra) mbar_arrive(&r_empty[sr]);
        }
        if (!extra && ++sr == kStagesR) sr = 0, pr ^= 1u;
        if (++sw == kStagesW) sw = 0, pw ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (M >= 256): a (2,1,1) cluster computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2, as the dense pair GEMM does.  Each CTA stages its
// own 128 rows of X and dequantises only its own 128 rows (forward) or output
// columns (backward) of the weight tile, so per SM the dequantisers convert
// half as many weights per k-block as in the one-CTA kernel, while the pair
// MMA reads half of B from each SM.  Sixteen dequantiser warps work in four
// groups on four k-blocks at once, k-block i into W stage i mod kStagesW;
// a 4-bit row goes through a register codebook (row_codebook / codebook8).
// NF4 11008 x 4096, r 64: 0.39-0.43 ms at 4096 tokens and 0.082-0.090 ms at
// 512; the staged path (one dequantisation pass, then the dense pair GEMM)
// stays faster at 4096 tokens (0.29 ms), where each weight is converted
// once per 256-token tile, 16 times.
//   even CTA: producer arms x_full[s] for both CTAs' X bytes; warp 1 issues the
//             MMAs once both CTAs' dequantisers have arrived on w_full[s], and
//             commits to both CTAs' x_empty / w_empty / acc_full.
//   odd CTA:  X copies complete on the even CTA's x_full; its dequantisers
//             arrive on the even CTA's w_full.
// Raw codes and scales go to each CTA's own ring, on its own barriers.
constexpr int kPHalf = 128;
constexpr int kPStagesX = 6;
constexpr int kPStagesR = 4;
// dequantiser warps of the pair kernel: four groups; each thread of a group
// converts 128 / (group threads) 64-weight rows per k-block
constexpr int kPDqWarps = 16;
constexpr int kPGroupThreads = 32 * kPDqWarps / 4;
constexpr int kPRowsPerThread = 128 / kPGroupThreads;
constexpr int kPThreads = 64 + 32 * kEpiWarps + 32 * kPDqWarps;
constexpr uint32_t kPXBytes = kPHalf * kBK * 2;  // 16 KB
constexpr uint32_t kPWBytes = kPHalf * kBK * 2;  // 16 KB

template <int kScheme>
struct QPairTraits {
  static constexpr int kBits = kScheme == kINT8 ? 8 : 4;
  // forward [128 rows x 64 k] or backward [64 rows x 128 columns] of codes
  static constexpr uint32_t kCodeBytes = kPHalf * kBK * kBits / 8;
  static constexpr uint32_t kScaleBytes = 1024;
  static constexpr uint32_t kRawBytes = kCodeBytes + kScaleBytes;
  // W stages, dealt round-robin (k-block i converts into stage i % kStagesW):
  // as many as the shared memory holds beside the X and raw rings
  static constexpr int kStagesW = kBits == 4 ? 6 : 5;
};

template <int kScheme>
constexpr size_t pair_smem_bytes() {
  return 1024 + kPStagesX * kPXBytes + QPairTraits<kScheme>::kStagesW * kPWBytes +
         kPStagesR * QPairTraits<kScheme>::kRawBytes + 512;
}

template <int kScheme, bool kWMN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    qlora_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_x,
                           const __grid_constant__ CUtensorMap tm_x2,
                           const __grid_constant__ CUtensorMap tm_codes,
                           const __grid_constant__ CUtensorMap tm_scales, const QGemmParams p) {
  using Tr = QPairTraits<kScheme>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint8_t* xs = smem;
  uint8_t* ws = xs + kPStagesX * kPXBytes;
  uint8_t* rs = ws + Tr::kStagesW * kPWBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(rs + kPStagesR * Tr::kRawBytes);
  uint64_t* x_full = bars;
  uint64_t* x_empty = x_full + kPStagesX;
  uint64_t* r_full = x_empty + kPStagesX;
  uint64_t* r_empty = r_full + kPStagesR;
  uint64_t* w_full = r_empty + kPStagesR;
  uint64_t* w_empty = w_full + Tr::kStagesW;
  uint64_t* acc_full = w_empty + Tr::kStagesW;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t crank = cluster_ctarank();
  const bool lead = crank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int num_pairs = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStagesX; ++s) mbar_init(&x_full[s], 1), mbar_init(&x_empty[s], 1);
    for (int s = 0; s < kPStagesR; ++s) mbar_init(&r_full[s], 1), mbar_init(&r_empty[s], 1);
    // the even CTA's w_full counts one arrival from each CTA's dequantisers
    for (int s = 0; s < Tr::kStagesW; ++s) mbar_init(&w_full[s], 2), mbar_init(&w_empty[s], 1);
    for (int b = 0; b < 2; ++b) mbar_init(&acc_full[b], 1), mbar_init(&acc_empty[b], 2 * kEpiWarps);
    mbar_init(drain_bar, 1);
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_codes);
    prefetch_tmap(&tm_scales);
    if (p.num_kb_extra > 0) prefetch_tmap(&tm_x2);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_kb = p.num_kb_main + p.num_kb_extra;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (elect_one()) {
      const uint32_t lead_xfull = mapa_shared(smem_u32(x_full), 0);
      uint32_t sx = 0, px = 0, sr = 0, pr = 0;
      bool armed_x[kPStagesX], armed_r[kPStagesR];
      uint32_t par_x[kPStagesX], par_r[kPStagesR];
      for (int s = 0; s < kPStagesX; ++s) armed_x[s] = false, par_x[s] = 0;
      for (int s = 0; s < kPStagesR; ++s) armed_r[s] = false, par_r[s] = 0;
      bool ok = true;
      for (int tile = pair; tile < p.num_tiles && ok; tile += num_pairs) {
        const int m0 = (tile / p.tiles_n) * (2 * kPHalf) + static_cast<int>(crank) * kPHalf;
        const int c0 = (tile % p.tiles_n) * (2 * kPHalf) + static_cast<int>(crank) * kPHalf;
        for (int kb = 0; kb < total_kb && ok; ++kb) {
          const bool extra = kb >= p.num_kb_main;
          if (!mbar_wait(&x_empty[sx], px ^ 1u, p.status, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (lead) {
            mbar_arrive_expect_tx(&x_full[sx], 2 * kPXBytes);
            armed_x[sx] = true;
            par_x[sx] = px;
          }
          const int k0 = (extra ? kb - p.num_kb_main : kb) * kBK;
          tma_load_2d_pair(xs + sx * kPXBytes, extra ? &tm_x2 : &tm_x, lead_xfull + sx * 8u, k0,
                           m0);
          if (++sx == kPStagesX) sx = 0, px ^= 1u;
          if (extra) continue;
          if (!mbar_wait(&r_empty[sr], pr ^ 1u, p.status, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* raw = rs + sr * Tr::kRawBytes;
          mbar_arrive_expect_tx(&r_full[sr], Tr::kCodeBytes + p.scale_box_bytes);
          armed_r[sr] = true;
          par_r[sr] = pr;
          if constexpr (kWMN) {
            // rows: the reduction index in [kb*64, kb*64+64); this CTA's 128 output columns
            tma_load_2d(raw, &tm_codes, &r_full[sr], c0 * Tr::kBits / 8, kb * kBK);
            tma_load_2d(raw + Tr::kCodeBytes, &tm_scales, &r_full[sr], kb * kBK, c0 / p.group);
          } else {
            tma_load_2d(raw, &tm_codes, &r_full[sr], kb * kBK * Tr::kBits / 8, c0);
            tma_load_2d(raw + Tr::kCodeBytes, &tm_scales, &r_full[sr], c0, (kb * kBK) / p.group);
          }
          if (++sr == kPStagesR) sr = 0, pr ^= 1u;
        }
      }
      // never leave a copy in flight at exit (the even CTA's x_full counts
      // both CTAs' X bytes; the raw copies land on this CTA's own barriers)
      for (int s = 0; s < kPStagesX; ++s)
        if (armed_x[s]) mbar_wait(&x_full[s], par_x[s], p.status, kDevTimeoutDrain);
      for (int s = 0; s < kPStagesR; ++s)
        if (armed_r[s]) mbar_wait(&r_full[s], par_r[s], p.status, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    // ------------------------------------------------- MMA (even CTA only) --
    if (lead && elect_one()) {
      constexpr uint32_t idesc = make_idesc_f16(2 * kPHalf, 2 * kPHalf, false, kWMN, true);
      const uint32_t peer_xempty = mapa_shared(smem_u32(x_empty), 1);
      const uint32_t peer_wempty = mapa_shared(smem_u32(w_empty), 1);
      const uint32_t peer_acc_full = mapa_shared(smem_u32(acc_full), 1);
      uint32_t sx = 0, px = 0, sw = 0, pw = 0;
      int local = 0;
      bool ok = true;
      for (int tile = pair; tile < p.num_tiles && ok; tile += num_pairs, ++local) {
        const uint32_t buf = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1) & 1u;
        if (!mbar_wait(&acc_empty[buf], use ^ 1u, p.status, kDevTimeoutAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * kBN;
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&x_full[sx], px, p.status, kDevTimeoutFull) ||
              !mbar_wait(&w_full[sw], pw, p.status, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sxa = smem_u32(xs + sx * kPXBytes);
          const uint32_t swa = smem_u32(ws + sw * kPWBytes);
          int nk = 4;
          if (kb >= p.num_kb_main) {
            const int rem = p.R - (kb - p.num_kb_main) * kBK;
            nk = rem >= kBK ? 4 : rem / 16;
          }
          for (int k = 0; k < nk; ++k) {
            uint64_t bd;
            if constexpr (kWMN)
              bd = desc_mnmajor_sw128(swa, k, kMNBoxBytes);
            else
              bd = desc_kmajor_sw128(swa, k);
            umma_f16_pair(d_tmem, desc_kmajor_sw128(sxa, k), bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(smem_u32(&x_empty[sx]));
          umma_commit_pair(peer_xempty + sx * 8u);
          umma_commit_pair(smem_u32(&w_empty[sw]));
          umma_commit_pair(peer_wempty + sw * 8u);
          if (++sx == kPStagesX) sx = 0, px ^= 1u;
          if (++sw == Tr::kStagesW) sw = 0, pw ^= 1u;
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&acc_full[buf]));
        umma_commit_pair(peer_acc_full + buf * 8u);
      }
      // every MMA issued above has completed before TMEM is released
      umma_commit_pair(smem_u32(drain_bar));
      mbar_wait(drain_bar, 0, p.status, kDevTimeoutDrain);
    }
  } else if (warp < 2 + kEpiWarps) {
    // ----------------------------------------------------------- epilogue --
    const uint32_t quarter = warp & 3u;
    const uint32_t row = quarter * 32 + lane;
    const uint32_t lead_acc_empty = mapa_shared(smem_u32(acc_empty), 0);
    const int vec = (p.N % 8 == 0 && p.ldd % 8 == 0) ? 1 : 0;
    int local = 0;
    for (int tile = pair; tile < p.num_tiles; tile += num_pairs, ++local) {
      const uint32_t buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1) & 1u;
      if (!mbar_wait(&acc_full[buf], use, p.status, kDevTimeoutAccFull)) break;
      tc_fence_after();
      const int m = (tile / p.tiles_n) * (2 * kPHalf) + static_cast<int>(crank) * kPHalf +
                    static_cast<int>(row);
      const int n_base = (tile % p.tiles_n) * (2 * kPHalf);
      __nv_bfloat16* out_row =
          reinterpret_cast<__nv_bfloat16*>(p.d) + static_cast<long long>(m) * p.ldd + n_base;
      const uint32_t taddr = tmem_base + ((quarter * 32u) << 16) + buf * kBN;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + c * 32, r);
        tmem_ld_wait();
        if (m < p.M) {
          const int n0 = n_base + c * 32;
          if (!vec) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (n0 + i < p.N) out_row[c * 32 + i] = __float2bfloat16_rn(__uint_as_float(r[i]));
            continue;
          }
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = pack2<__nv_bfloat16>(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (n0 + q * 8 < p.N)
              *reinterpret_cast<uint4*>(out_row + c * 32 + q * 8) =
                  make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(lead_acc_empty + buf * 8u);
    }
  } else {
    // -------------------------------------------------------- dequantisers --
    // Four groups; group g converts the k-blocks whose running index is g
    // (mod 4), k-block i into W stage i % 6, so four k-blocks are in
    // conversion at once and six are buffered.  A group waits only for stages
    // of earlier k-blocks, so the order is deadlock-free.  Work item w = u + kPGroupThreads * i0 of a group's 128: forward
    // row w of this CTA's 128; backward row w % 64 of 64-column box w / 64.
    const uint32_t t = threadIdx.x - (64 + 32 * kEpiWarps);
    const uint32_t grp = t / kPGroupThreads, u = t % kPGroupThreads;
    const uint32_t lead_wfull = mapa_shared(smem_u32(w_full), 0);
    uint32_t sr = 0, pr = 0, it = 0;
    bool ok = true;
    for (int tile = pair; tile < p.num_tiles && ok; tile += num_pairs) {
      const int c0 = (tile % p.tiles_n) * (2 * kPHalf) + static_cast<int>(crank) * kPHalf;
      for (int kb = 0; kb < total_kb; ++kb, ++it) {
        const bool extra = kb >= p.num_kb_main;
        const uint32_t my_sr = sr, my_pr = pr;
        if (!extra && ++sr == kPStagesR) sr = 0, pr ^= 1u;
        if ((it & 3u) != grp) continue;
        const uint32_t sw = it % Tr::kStagesW, pw = (it / Tr::kStagesW) & 1u;
        if (!mbar_wait(&w_empty[sw], pw ^ 1u, p.status, kDevTimeoutEmpty)) {
          ok = false;
          break;
        }
        uint8_t* wtile = ws + sw * kPWBytes;
        if (!extra) {
          if (!mbar_wait(&r_full[my_sr], my_pr, p.status, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          const uint8_t* raw = rs + my_sr * Tr::kRawBytes;
          const uint8_t* scales = raw + Tr::kCodeBytes;
#pragma unroll
          for (uint32_t i0 = 0; i0 < kPRowsPerThread; ++i0) {
            const uint32_t w = u + kPGroupThreads * i0;
            float s, z;
            if constexpr (kWMN) {
              const uint32_t i = w >> 6, uu = w & 63u;
              const uint32_t g = (static_cast<uint32_t>(c0) + i * 64u) / static_cast<uint32_t>(p.group) -
                                 static_cast<uint32_t>(c0) / static_cast<uint32_t>(p.group);
              scale_zero<kScheme>(scales, g * 64u + uu, s, z);
              dequant_row<kScheme>(raw + uu * (kPHalf * Tr::kBits / 8) + i * (64 * Tr::kBits / 8),
                                   s, z, wtile + i * kMNBoxBytes + uu * 128u, uu);
            } else {
              const uint32_t row = w;
              scale_zero<kScheme>(scales, row, s, z);
              dequant_row<kScheme>(raw + row * (kBK * Tr::kBits / 8), s, z, wtile + row * 128u,
                                   row);
            }
          }
        } else {
          // rank block: 64 columns of the up-projection operand (zero padded)
          const int j0 = (kb - p.num_kb_main) * kBK;
#pragma unroll
          for (uint32_t i0 = 0; i0 < kPRowsPerThread; ++i0) {
            const uint32_t w = u + kPGroupThreads * i0;
            if constexpr (kWMN) {
              const uint32_t i = w >> 6, uu = w & 63u;
              const int j = j0 + static_cast<int>(uu);
              uint8_t* out_row = wtile + i * kMNBoxBytes + uu * 128u;
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                const long long col = c0 + i * 64 + c * 8;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (j < p.up_rows && col < p.up_cols)
                  v = *reinterpret_cast<const uint4*>(p.up + static_cast<long long>(j) * p.up_ld + col);
                st_chunk(out_row, uu, c, v);
              }
            } else {
              const uint32_t row = w;
              const long long n = c0 + static_cast<long long>(row);
              uint8_t* out_row = wtile + row * 128u;
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                const int j = j0 + c * 8;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (n < p.N && j < p.up_rows)
                  v = *reinterpret_cast<const uint4*>(p.up + n * p.up_ld + j);
                st_chunk(out_row, row, c, v);
              }
            }
          }
        }
        fence_proxy_async_smem();
        named_bar_sync(2 + grp, kPGroupThreads);
        if (u == 0) {
          mbar_arrive_cluster(lead_wfull + sw * 8u);
          if (!extra) mbar_arrive(&r_empty[my_sr]);
        }
      }
    }
  }

  // After a failure the odd CTA may still have copies in flight that no
  // barrier of its own tracks: give them time to land before the pair exits.
  if (p.status != nullptr && *reinterpret_cast<volatile uint32_t*>(p.status) != 0) {
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 200000ull) {
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no arrival, copy or MMA of the other CTA still targets this one
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

bool make_tmap_raw(CUtensorMap* map, CUtensorMapDataType dt, uint32_t esize, const void* base,
                   uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                   uint32_t box_outer);

template <int kScheme, bool kWMN>
int launch_q(const QGemmArgs& a, cudaStream_t stream) {
  using Tr = QTraits<kScheme>;
  CUtensorMap tx, tx2, tc, ts;
  if (!make_tmap_2d_16b(&tx, a.x, a.K, a.M, a.ldx, kBK, kBM)) return MLORA_ERR_INVALID_ARG;
  if (a.R > 0) {
    const int64_t r64 = (a.R + 63) / 64 * 64;
    if (!make_tmap_2d_16b(&tx2, a.x2, r64, a.M, a.ldx2, kBK, kBM)) return MLORA_ERR_INVALID_ARG;
  } else {
    tx2 = tx;
  }
  // W geometry: forward: W rows = N (out), cols = K (in); backward: W rows = K_red, cols = N_out.
  const int64_t w_rows = kWMN ? a.K : a.N;
  const int64_t w_cols = kWMN ? a.N : a.K;
  const int64_t code_cols = w_cols * Tr::kBits / 8;  // bytes per W row
  const int64_t ngroups = (w_cols + a.group - 1) / a.group;
  uint32_t scale_box_bytes;
  if (kWMN) {
    if (!make_tmap_raw(&tc, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.codes, code_cols, w_rows,
                       code_cols, kBN * Tr::kBits / 8, kBK))
      return MLORA_ERR_INVALID_ARG;
    // scales_t [ngroups, w_rows]: box (64 rows of this k-block, the groups of 256 out-features)
    const uint32_t gbox = static_cast<uint32_t>(kBN / a.group);
    if (!make_tmap_raw(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, a.scales_t, w_rows, ngroups,
                       prepared_ld(w_rows) * 4, kBK, gbox))
      return MLORA_ERR_INVALID_ARG;
    scale_box_bytes = kBK * gbox * 4;
  } else {
    if (!make_tmap_raw(&tc, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.codes, code_cols, w_rows,
                       code_cols, kBK * Tr::kBits / 8, kBN))
      return MLORA_ERR_INVALID_ARG;
    if (!make_tmap_raw(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, a.scales_t, w_rows, ngroups,
                       prepared_ld(w_rows) * 4, kBN, 1))
      return MLORA_ERR_INVALID_ARG;
    scale_box_bytes = kBN * 4;
  }
  QGemmParams p;
  p.M = static_cast<int>(a.M);
  p.N = static_cast<int>(a.N);
  p.num_kb_main = static_cast<int>((a.K + kBK - 1) / kBK);
  p.R = static_cast<int>(a.R);
  p.num_kb_extra = static_cast<int>((a.R + kBK - 1) / kBK);
  const int tiles_m = static_cast<int>((a.M + kBM - 1) / kBM);
  p.tiles_n = static_cast<int>((a.N + kBN - 1) / kBN);
  p.num_tiles = tiles_m * p.tiles_n;
  p.group = static_cast<int>(a.group);
  p.scale_box_bytes = scale_box_bytes;
  p.d = a.d;
  p.ldd = a.ldd;
  p.up = static_cast<const __nv_bfloat16*>(a.up);
  p.up_rows = static_cast<int>(a.up_rows);
  p.up_ld = a.up_ld;
  p.up_cols = a.up_cols;
  p.status = device_status_ptr();

  auto kern = qlora_gemm_kernel<kScheme, kWMN>;
  constexpr size_t smem = smem_bytes<kScheme>();
  static_assert(smem <= 232448, "rings exceed the 227 KB of shared memory per CTA");
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) {
    set_error(std::string("cudaFuncSetAttribute(qgemm): ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
  LaunchScope scope(kKindGemm, stream);
  kern<<<grid, kThreads, smem, stream>>>(tx, tx2, tc, ts, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("qgemm launch: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

template <int kScheme, bool kWMN>
int launch_q_pair(const QGemmArgs& a, cudaStream_t stream) {
  using Tr = QPairTraits<kScheme>;
  CUtensorMap tx, tx2, tc, ts;
  if (!make_tmap_2d_16b(&tx, a.x, a.K, a.M, a.ldx, kBK, kPHalf)) return MLORA_ERR_INVALID_ARG;
  if (a.R > 0) {
    const int64_t r64 = (a.R + 63) / 64 * 64;
    if (!make_tmap_2d_16b(&tx2, a.x2, r64, a.M, a.ldx2, kBK, kPHalf)) return MLORA_ERR_INVALID_ARG;
  } else {
    tx2 = tx;
  }
  // W geometry: forward: W rows = N (out), cols = K (in); backward: W rows = K_red, cols = N_out.
  const int64_t w_rows = kWMN ? a.K : a.N;
  const int64_t w_cols = kWMN ? a.N : a.K;
  const int64_t code_cols = w_cols * Tr::kBits / 8;  // bytes per W row
  const int64_t ngroups = (w_cols + a.group - 1) / a.group;
  uint32_t scale_box_bytes;
  if (kWMN) {
    // codes: 64 reduction rows x this CTA's 128 output columns
    if (!make_tmap_raw(&tc, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.codes, code_cols, w_rows,
                       code_cols, kPHalf * Tr::kBits / 8, kBK))
      return MLORA_ERR_INVALID_ARG;
    const uint32_t gbox = a.group >= kPHalf ? 1u : static_cast<uint32_t>(kPHalf / a.group);
    if (!make_tmap_raw(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, a.scales_t, w_rows, ngroups,
                       prepared_ld(w_rows) * 4, kBK, gbox))
      return MLORA_ERR_INVALID_ARG;
    scale_box_bytes = kBK * gbox * 4;
  } else {
    // codes: this CTA's 128 rows x 64 k
    if (!make_tmap_raw(&tc, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.codes, code_cols, w_rows,
                       code_cols, kBK * Tr::kBits / 8, kPHalf))
      return MLORA_ERR_INVALID_ARG;
    if (!make_tmap_raw(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, a.scales_t, w_rows, ngroups,
                       prepared_ld(w_rows) * 4, kPHalf, 1))
      return MLORA_ERR_INVALID_ARG;
    scale_box_bytes = kPHalf * 4;
  }
  if (scale_box_bytes > Tr::kScaleBytes) {
    set_error("qgemm pair: scale groups too small for the staged scale box");
    return MLORA_ERR_UNSUPPORTED;
  }
  QGemmParams p;
  p.M = static_cast<int>(a.M);
  p.N = static_cast<int>(a.N);
  p.num_kb_main = static_cast<int>((a.K + kBK - 1) / kBK);
  p.R = static_cast<int>(a.R);
  p.num_kb_extra = static_cast<int>((a.R + kBK - 1) / kBK);
  const int tiles_m = static_cast<int>((a.M + 2 * kPHalf - 1) / (2 * kPHalf));
  p.tiles_n = static_cast<int>((a.N + 2 * kPHalf - 1) / (2 * kPHalf));
  p.num_tiles = tiles_m * p.tiles_n;
  p.group = static_cast<int>(a.group);
  p.scale_box_bytes = scale_box_bytes;
  p.d = a.d;
  p.ldd = a.ldd;
  p.up = static_cast<const __nv_bfloat16*>(a.up);
  p.up_rows = static_cast<int>(a.up_rows);
  p.up_ld = a.up_ld;
  p.up_cols = a.up_cols;
  p.status = device_status_ptr();

  auto kern = qlora_gemm_pair_kernel<kScheme, kWMN>;
  constexpr size_t smem = pair_smem_bytes<kScheme>();
  static_assert(smem <= 232448, "pair kernel rings exceed the 227 KB of shared memory per CTA");
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) {
    set_error(std::string("cudaFuncSetAttribute(qgemm pair): ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  const int pairs = std::min(p.num_tiles, num_sms() / 2);
  LaunchScope scope(kKindGemm, stream);
  kern<<<2 * pairs, kPThreads, smem, stream>>>(tx, tx2, tc, ts, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("qgemm pair launch: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

bool make_tmap_raw(CUtensorMap* map, CUtensorMapDataType dt, uint32_t esize, const void* base,
                   uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                   uint32_t box_outer) {
  return make_tmap_2d(map, dt, esize, base, inner, outer, row_stride_bytes, box_inner, box_outer,
                      false);
}

}  // namespace

// The CTA-pair kernel serves M >= 256 unless MLORA_GEMM_PAIR=0; both give the
// same results (the same bf16 weights, the same per-tile reduction order).
bool qpair_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MLORA_GEMM_PAIR");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}

int launch_qgemm(const QGemmArgs& a, cudaStream_t stream) {
  if (a.M >= 2 * kPHalf && qpair_enabled()) {
    switch (a.scheme) {
      case kNF4: return a.w_mn_major ? launch_q_pair<kNF4, true>(a, stream) : launch_q_pair<kNF4, false>(a, stream);
      case kINT4: return a.w_mn_major ? launch_q_pair<kINT4, true>(a, stream) : launch_q_pair<kINT4, false>(a, stream);
      case kINT8: return a.w_mn_major ? launch_q_pair<kINT8, true>(a, stream) : launch_q_pair<kINT8, false>(a, stream);
      default: break;
    }
  }
  switch (a.scheme) {
    case kNF4: return a.w_mn_major ? launch_q<kNF4, true>(a, stream) : launch_q<kNF4, false>(a, stream);
    case kINT4: return a.w_mn_major ? launch_q<kINT4, true>(a, stream) : launch_q<kINT4, false>(a, stream);
    case kINT8: return a.w_mn_major ? launch_q<kINT8, true>(a, stream) : launch_q<kINT8, false>(a, stream);
    default: set_error("unknown quantisation scheme"); return MLORA_ERR_INVALID_ARG;
  }
}

}  // namespace mlora
