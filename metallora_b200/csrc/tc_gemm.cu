// Persistent tcgen05 GEMM with an appended rank-r block:
//
//     D[M, N] = X[M, K] . W^T  +  X2[M, R] . W2^T
//
// It serves both dense LoRA-linear GEMMs:
//   forward  y  = x . W0^T + (s x A^T) . B^T        X = x,  W = W0 (K-major), X2 = s.x.A^T, W2 = B
//   backward dx = dy . W0  + (s dy B) . A           X = dy, W = W0 (MN-major), X2 = s.dy.B, W2 = A
// (reference math: python/metal_lora/ops.py:91-94 and its chain rule).  The rank-r
// block is just R/16 more UMMA k-steps into the same TMEM accumulator, so D is
// written exactly once.
//
// Structure (one CTA per SM, 6 warps):
//   warp 0     TMA producer (one elected lane): X tile [128 x 64] and W tile
//              [256 x 64] per stage, 128-byte swizzle, mbarrier tx accounting.
//   warp 1     TMEM allocator + UMMA issuer (one elected lane): M=128, N=256,
//              K=16 per instruction, fp32 accumulators double-buffered in TMEM
//              (2 x 256 of the 512 columns) so the epilogue of tile i overlaps
//              the main loop of tile i+1.
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time, convert, 16-byte
//              global stores; each thread owns one output row.
// Tiles are visited n-fastest so the CTAs resident at one time share W and X
// tiles in L2.
#include <atomic>
#include <cstdlib>
#include <string>

#include "internal.h"
#include "ptx.cuh"
#include "../../include/metallora_b200.h"

namespace mlora {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr uint32_t kXTileBytes = kBM * kBK * 2;  // 16 KB
constexpr uint32_t kWTileBytes = kBN * kBK * 2;  // 32 KB
constexpr uint32_t kStageBytes = kXTileBytes + kWTileBytes;
constexpr uint32_t kMNBoxBytes = 64 * kBK * 2;   // one MN-major TMA box (8 KB)
constexpr int kEpiWarps = 4;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t kTmemCols = 512;
constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + 256;

struct GemmParams {
  int M, N;
  int num_kb_main, num_kb_extra, R;
  int tiles_m, tiles_n, num_tiles;
  int group_m;  // tile rows per raster group
  int wait_prev;  // programmatic dependent: wait for the previous grid before X2 loads
  void* d;
  long long ldd;
  const void* c;  // optional addend, same type/layout as d (ldc)
  long long ldc;
  const int32_t* c_index;  // optional: addend row of output row m is c_index[m] (< c_rows)
  long long c_rows;
  float acc_scale;
  int vec_ok;     // rows of d (and c) allow 16-byte vector access
  uint32_t* status;
};

// Tile order: groups of `group_m` tile rows; inside a group, tile rows vary
// fastest and tile columns sweep across N.  The tiles resident at one time then
// cover a compact block (group_m rows x a few columns), so each W tile is read
// from HBM about once per group and each X tile once overall, even when W is
// larger than L2 (plain column-fastest order re-reads all of W for every few
// tile rows once W no longer fits).
__device__ __forceinline__ void tile_coords(const GemmParams& p, int tile, int& tm, int& tn) {
  const int per_group = p.group_m * p.tiles_n;
  const int g = tile / per_group;
  const int rem = tile - g * per_group;
  const int rows = min(p.group_m, p.tiles_m - g * p.group_m);
  tm = g * p.group_m + rem % rows;
  tn = rem / rows;
}

// Epilogue of one accumulator row: this thread's output row m, columns
// [n_base, n_base + 256), from TMEM at `taddr` (its lane, the buffer's first
// column).  Scales by acc_scale, adds the optional (row-gathered) addend,
// converts and stores with 16-byte vectors when rows allow.
template <typename OutT>
__device__ __forceinline__ void store_row(const GemmParams& p, int m, int n_base, uint32_t taddr) {
  OutT* out_row = reinterpret_cast<OutT*>(p.d) + static_cast<long long>(m) * p.ldd + n_base;
  // the addend's row: m, or a gathered row (an index outside the table
  // contributes nothing and is reported in the status word)
  const OutT* c_row = nullptr;
  if (p.c != nullptr && m < p.M) {
    long long cr = m;
    if (p.c_index != nullptr) {
      cr = p.c_index[m];
      if (cr < 0 || cr >= p.c_rows) {
        record_status(p.status, kDevBadIndex);
        cr = -1;
      }
    }
    if (cr >= 0) c_row = reinterpret_cast<const OutT*>(p.c) + cr * p.ldc + n_base;
  }
#pragma unroll 1
  for (int c = 0; c < kBN / 32; ++c) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr + c * 32, r);
    tmem_ld_wait();
    if (m < p.M) {
      const int n0 = n_base + c * 32;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * p.acc_scale;
      if (!p.vec_ok) {
        // ragged or unaligned rows: element-wise, bounds-checked
        const OutT* crow = c_row != nullptr ? c_row + c * 32 : nullptr;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (n0 + i < p.N) {
            float o = v[i];
            if (crow != nullptr) o += static_cast<float>(crow[i]);
            out_row[c * 32 + i] = static_cast<OutT>(o);
          }
        }
        continue;
      }
      if (c_row != nullptr) {
        const OutT* crow = c_row + c * 32;
        if constexpr (sizeof(OutT) == 2) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (n0 + q * 8 < p.N) {
              const uint4 cv = *reinterpret_cast<const uint4*>(crow + q * 8);
              const OutT* ce = reinterpret_cast<const OutT*>(&cv);
#pragma unroll
              for (int i = 0; i < 8; ++i) v[q * 8 + i] += static_cast<float>(ce[i]);
            }
          }
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            if (n0 + q * 4 < p.N) {
              const float4 cv = *reinterpret_cast<const float4*>(crow + q * 4);
              v[q * 4] += cv.x;
              v[q * 4 + 1] += cv.y;
              v[q * 4 + 2] += cv.z;
              v[q * 4 + 3] += cv.w;
            }
          }
        }
      }
      if constexpr (sizeof(OutT) == 2) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack2<OutT>(v[2 * i], v[2 * i + 1]);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (n0 + q * 8 < p.N)
            *reinterpret_cast<uint4*>(out_row + c * 32 + q * 8) =
                make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (n0 + q * 4 < p.N)
            *reinterpret_cast<float4*>(out_row + c * 32 + q * 4) =
                make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      }
    }
  }
}

template <bool kWMN, bool kBF16, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    lora_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_x2,
                     const __grid_constant__ CUtensorMap tm_w2, const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* acc_full = empty_bar + kStages;   // [2]
  uint64_t* acc_empty = acc_full + 2;         // [2]
  uint64_t* drain_bar = acc_empty + 2;        // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps * 32);
    }
    mbar_init(drain_bar, 1);
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
    if (p.num_kb_extra > 0) {
      prefetch_tmap(&tm_x2);
      prefetch_tmap(&tm_w2);
    }
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
      uint32_t stage = 0, phase = 0;
      uint32_t armed_parity[kStages];
      bool armed[kStages];
      for (int s = 0; s < kStages; ++s) armed[s] = false, armed_parity[s] = 0;
      bool ok = true;
      bool prev_done = false;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int tm, tn;
        tile_coords(p, tile, tm, tn);
        const int m0 = tm * kBM;
        const int n0 = tn * kBN;
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, p.status, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sx = smem + stage * kStageBytes;
          uint8_t* sw = sx + kXTileBytes;
          mbar_arrive_expect_tx(&full_bar[stage], kStageBytes);
          armed[stage] = true;
          armed_parity[stage] = phase;
          const bool extra = kb >= p.num_kb_main;
          if (extra && p.wait_prev && !prev_done) {  // X2 comes from the previous grid
            asm volatile("griddepcontrol.wait;" ::: "memory");
            prev_done = true;
          }
          const CUtensorMap* mx = extra ? &tm_x2 : &tm_x;
          const CUtensorMap* mw = extra ? &tm_w2 : &tm_w;
          const int k0 = (extra ? kb - p.num_kb_main : kb) * kBK;
          tma_load_2d(sx, mx, &full_bar[stage], k0, m0);
          if constexpr (kWMN) {
#pragma unroll
            for (int i = 0; i < kBN / 64; ++i)
              tma_load_2d(sw + i * kMNBoxBytes, mw, &full_bar[stage], n0 + i * 64, k0);
          } else {
            tma_load_2d(sw, mw, &full_bar[stage], k0, n0);
          }
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
      }
      // Never leave a bulk copy in flight at exit.
      for (int s = 0; s < kStages; ++s)
        if (armed[s]) mbar_wait(&full_bar[s], armed_parity[s], p.status, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA --
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_f16(kBM, kBN, false, kWMN, kBF16);
      uint32_t stage = 0, phase = 0;
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
          if (!mbar_wait(&full_bar[stage], phase, p.status, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sx = smem_u32(smem + stage * kStageBytes);
          const uint32_t sw = sx + kXTileBytes;
          int nk = 4;
          if (kb >= p.num_kb_main) {
            const int rem = p.R - (kb - p.num_kb_main) * kBK;
            nk = rem >= kBK ? 4 : rem / 16;
          }
          for (int k = 0; k < nk; ++k) {
            const uint64_t ad = desc_kmajor_sw128(sx, k);
            uint64_t bd;
            if constexpr (kWMN)
              bd = desc_mnmajor_sw128(sw, k, kMNBoxBytes);
            else
              bd = desc_kmajor_sw128(sw, k);
            umma_f16(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
      }
      // Drain: every UMMA issued above has completed before TMEM is released.
      umma_commit(drain_bar);
      mbar_wait(drain_bar, 0, p.status, kDevTimeoutDrain);
    }
  } else {
    // ----------------------------------------------------------- epilogue --
    const uint32_t quarter = warp & 3u;  // TMEM lanes [32*quarter, 32*quarter+32)
    const uint32_t row = quarter * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      const uint32_t buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1) & 1u;
      if (!mbar_wait(&acc_full[buf], use, p.status, kDevTimeoutAccFull)) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(p, tile, tm, tn);
      const int m = tm * kBM + static_cast<int>(row);
      const int n_base = tn * kBN;
      const uint32_t taddr = tmem_base + ((quarter * 32u) << 16) + buf * kBN;
      store_row<OutT>(p, m, n_base, taddr);
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
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
// CTA-pair variant: a (2,1,1) cluster computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16).  Each CTA stages its own
// 128 rows of X and 128 rows (columns of D) of W per k-block, so per MMA
// cycle each SM's shared memory feeds half of B instead of all of it, and
// each CTA loads 32 KB per stage instead of 48 KB.  Each CTA's TMEM holds its
// 128 rows of the accumulator (2 x 256 columns, double-buffered) and its own
// epilogue stores them.
//   even CTA: producer arms full[s] for both CTAs' bytes; warp 1 issues the
//             MMAs and commits to both CTAs' empty[s] / acc_full[b];
//             acc_empty[b] counts 4 epilogue warps of each CTA.
//   odd CTA:  producer waits its own empty[s] and loads with completion on
//             the even CTA's full[s]; epilogue as the even CTA's.
// Every copy lands in the shared memory of the CTA that issues it.
constexpr int kPairStages = 6;
constexpr int kHalf = 128;                                // rows of X / W per CTA
constexpr uint32_t kPairXBytes = kHalf * kBK * 2;         // 16 KB
constexpr uint32_t kPairWBytes = kHalf * kBK * 2;         // 16 KB
constexpr uint32_t kPairStageBytes = kPairXBytes + kPairWBytes;
constexpr size_t kPairSmemBytes = 1024 + kPairStages * kPairStageBytes + 256;

template <bool kWMN, bool kBF16, typename OutT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    lora_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_x,
                          const __grid_constant__ CUtensorMap tm_w,
                          const __grid_constant__ CUtensorMap tm_x2,
                          const __grid_constant__ CUtensorMap tm_w2, const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kPairStages * kPairStageBytes);
  uint64_t* empty_bar = full_bar + kPairStages;
  uint64_t* acc_full = empty_bar + kPairStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;            // [2]
  uint64_t* drain_bar = acc_empty + 2;           // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t crank = cluster_ctarank();
  const bool lead = crank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int num_pairs = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
    if (p.num_kb_extra > 0) {
      prefetch_tmap(&tm_x2);
      prefetch_tmap(&tm_w2);
    }
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
      const uint32_t lead_full = mapa_shared(smem_u32(full_bar), 0);
      uint32_t stage = 0, phase = 0;
      uint32_t armed_parity[kPairStages];
      bool armed[kPairStages];
      for (int s = 0; s < kPairStages; ++s) armed[s] = false, armed_parity[s] = 0;
      bool ok = true;
      bool prev_done = false;
      for (int tile = pair; tile < p.num_tiles && ok; tile += num_pairs) {
        int tm, tn;
        tile_coords(p, tile, tm, tn);
        const int m0 = tm * (2 * kHalf) + static_cast<int>(crank) * kHalf;
        const int n0 = tn * (2 * kHalf) + static_cast<int>(crank) * kHalf;
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, p.status, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sx = smem + stage * kPairStageBytes;
          uint8_t* sw = sx + kPairXBytes;
          if (lead) {
            mbar_arrive_expect_tx(&full_bar[stage], 2 * kPairStageBytes);
            armed[stage] = true;
            armed_parity[stage] = phase;
          }
          const uint32_t bar = lead_full + stage * 8u;
          const bool extra = kb >= p.num_kb_main;
          if (extra && p.wait_prev && !prev_done) {  // X2 comes from the previous grid
            asm volatile("griddepcontrol.wait;" ::: "memory");
            prev_done = true;
          }
          const CUtensorMap* mx = extra ? &tm_x2 : &tm_x;
          const CUtensorMap* mw = extra ? &tm_w2 : &tm_w;
          const int k0 = (extra ? kb - p.num_kb_main : kb) * kBK;
          tma_load_2d_pair(sx, mx, bar, k0, m0);
          if constexpr (kWMN) {
#pragma unroll
            for (int i = 0; i < kHalf / 64; ++i)
              tma_load_2d_pair(sw + i * kMNBoxBytes, mw, bar, n0 + i * 64, k0);
          } else {
            tma_load_2d_pair(sw, mw, bar, k0, n0);
          }
          if (++stage == kPairStages) stage = 0, phase ^= 1u;
        }
      }
      // Never leave a copy in flight at exit (the even CTA's barriers count
      // both CTAs' bytes).
      for (int s = 0; s < kPairStages; ++s)
        if (armed[s]) mbar_wait(&full_bar[s], armed_parity[s], p.status, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    // ------------------------------------------------- MMA (even CTA only) --
    if (lead && elect_one()) {
      constexpr uint32_t idesc = make_idesc_f16(2 * kHalf, 2 * kHalf, false, kWMN, kBF16);
      const uint32_t peer_empty = mapa_shared(smem_u32(empty_bar), 1);
      const uint32_t peer_acc_full = mapa_shared(smem_u32(acc_full), 1);
      uint32_t stage = 0, phase = 0;
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
          if (!mbar_wait(&full_bar[stage], phase, p.status, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sx = smem_u32(smem + stage * kPairStageBytes);
          const uint32_t sw = sx + kPairXBytes;
          int nk = 4;
          if (kb >= p.num_kb_main) {
            const int rem = p.R - (kb - p.num_kb_main) * kBK;
            nk = rem >= kBK ? 4 : rem / 16;
          }
          for (int k = 0; k < nk; ++k) {
            const uint64_t ad = desc_kmajor_sw128(sx, k);
            uint64_t bd;
            if constexpr (kWMN)
              bd = desc_mnmajor_sw128(sw, k, kMNBoxBytes);
            else
              bd = desc_kmajor_sw128(sw, k);
            umma_f16_pair(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(smem_u32(&empty_bar[stage]));
          umma_commit_pair(peer_empty + stage * 8u);
          if (++stage == kPairStages) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&acc_full[buf]));
        umma_commit_pair(peer_acc_full + buf * 8u);
      }
      // Drain: every MMA issued above has completed before TMEM is released.
      umma_commit_pair(smem_u32(drain_bar));
      mbar_wait(drain_bar, 0, p.status, kDevTimeoutDrain);
    }
  } else {
    // ----------------------------------------------------------- epilogue --
    const uint32_t quarter = warp & 3u;  // TMEM lanes [32*quarter, 32*quarter+32)
    const uint32_t row = quarter * 32 + lane;
    const uint32_t lead_acc_empty = mapa_shared(smem_u32(acc_empty), 0);
    int local = 0;
    for (int tile = pair; tile < p.num_tiles; tile += num_pairs, ++local) {
      const uint32_t buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1) & 1u;
      if (!mbar_wait(&acc_full[buf], use, p.status, kDevTimeoutAccFull)) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(p, tile, tm, tn);
      const int m = tm * (2 * kHalf) + static_cast<int>(crank) * kHalf + static_cast<int>(row);
      const int n_base = tn * (2 * kHalf);
      const uint32_t taddr = tmem_base + ((quarter * 32u) << 16) + buf * kBN;
      store_row<OutT>(p, m, n_base, taddr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(lead_acc_empty + buf * 8u);
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
  cluster_sync();  // no arrival or copy from the other CTA is still pending
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// The CTA-pair kernel is used from M >= 256 unless MLORA_GEMM_PAIR=0 (the
// single-CTA kernel then serves every size; both give the same results).
bool pair_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MLORA_GEMM_PAIR");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}

// Plain launch, or a programmatic dependent launch of the previous kernel on
// the stream (`dependent`).
template <typename Kern>
cudaError_t launch_maybe_dependent(Kern kern, int grid, size_t smem, cudaStream_t stream, bool dependent,
                            const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& tx2,
                            const CUtensorMap& tw2, const GemmParams& p) {
  if (!dependent) {
    kern<<<grid, kThreads, smem, stream>>>(tx, tw, tx2, tw2, p);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tx, tw, tx2, tw2, p);
  return e == cudaSuccess ? cudaGetLastError() : e;
}

// `done`: per-device flags (atomic: host threads may launch concurrently; a
// repeated cudaFuncSetAttribute with the same value is harmless)
template <typename Kern>
int set_smem_attr(Kern kern, size_t bytes, std::atomic<bool>* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !done[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(bytes));
    if (e != cudaSuccess) {
      set_error(std::string("cudaFuncSetAttribute(gemm): ") + cudaGetErrorString(e));
      return MLORA_ERR_CUDA;
    }
    if (dev < 64) done[dev].store(true, std::memory_order_release);
  }
  return MLORA_OK;
}

template <bool kWMN, bool kBF16, typename OutT>
int launch_typed(const GemmArgs& a, cudaStream_t stream) {
  const bool pair = a.M >= 2 * kHalf && pair_enabled();
  const int w_box_rows = pair ? kHalf : kBN;  // K-major W rows per CTA
  const int tile_m = pair ? 2 * kHalf : kBM, tile_n = pair ? 2 * kHalf : kBN;
  CUtensorMap tx, tw, tx2, tw2;
  if (!make_tmap_2d_16b(&tx, a.x, a.K, a.M, a.ldx, kBK, kBM)) return MLORA_ERR_INVALID_ARG;
  if (kWMN) {
    if (!make_tmap_2d_16b(&tw, a.w, a.N, a.K, a.ldw, 64, kBK)) return MLORA_ERR_INVALID_ARG;
  } else {
    if (!make_tmap_2d_16b(&tw, a.w, a.K, a.N, a.ldw, kBK, w_box_rows)) return MLORA_ERR_INVALID_ARG;
  }
  if (a.R > 0) {
    const int64_t r64 = (a.R + 63) / 64 * 64;
    if (!make_tmap_2d_16b(&tx2, a.x2, r64, a.M, a.ldx2, kBK, kBM)) return MLORA_ERR_INVALID_ARG;
    if (kWMN) {
      if (!make_tmap_2d_16b(&tw2, a.w2, a.N, a.w2_rows, a.ldw2, 64, kBK))
        return MLORA_ERR_INVALID_ARG;
    } else {
      if (!make_tmap_2d_16b(&tw2, a.w2, a.w2_rows, a.N, a.ldw2, kBK, w_box_rows))
        return MLORA_ERR_INVALID_ARG;
    }
  } else {
    tx2 = tx;
    tw2 = tw;
  }
  GemmParams p;
  p.M = static_cast<int>(a.M);
  p.N = static_cast<int>(a.N);
  p.num_kb_main = static_cast<int>((a.K + kBK - 1) / kBK);
  p.R = static_cast<int>(a.R);
  p.num_kb_extra = static_cast<int>((a.R + kBK - 1) / kBK);
  const int tiles_m = static_cast<int>((a.M + tile_m - 1) / tile_m);
  p.tiles_m = tiles_m;
  p.tiles_n = static_cast<int>((a.N + tile_n - 1) / tile_n);
  p.num_tiles = tiles_m * p.tiles_n;
  // W that stays in L2 next to the X tiles in use: column-fastest order (measured
  // best, e.g. 16384 x 4096 x 4096: 1558 vs 1520 TFLOP/s); larger W: raster
  // groups of 2048 rows of X (4096 x 4096 x 14336: 1446 vs 1251 TFLOP/s)
  const int64_t w_bytes = a.N * a.K * 2;
  const int group = w_bytes <= (int64_t{48} << 20) ? 1 : (pair ? 8 : 16);
  p.group_m = group < tiles_m ? group : tiles_m;
  p.d = a.d;
  p.ldd = a.ldd;
  p.c = a.c;
  p.ldc = a.ldc;
  p.c_index = a.c_index;
  p.c_rows = a.c_rows;
  p.acc_scale = a.acc_scale;
  p.wait_prev = (a.overlap_prev && a.R > 0) ? 1 : 0;
  {
    const int64_t vec = 16 / static_cast<int64_t>(sizeof(OutT));
    const bool d_ok = a.N % vec == 0 && a.ldd % vec == 0 &&
                      (reinterpret_cast<uintptr_t>(a.d) & 15u) == 0;
    const bool c_ok = a.c == nullptr ||
                      (a.ldc % vec == 0 && (reinterpret_cast<uintptr_t>(a.c) & 15u) == 0);
    p.vec_ok = (d_ok && c_ok) ? 1 : 0;
  }
  p.status = device_status_ptr();

  int rc;
  cudaError_t err = cudaSuccess;
  if (pair) {
    auto kern = lora_gemm_pair_kernel<kWMN, kBF16, OutT>;
    static std::atomic<bool> attr_set[64];
    static std::atomic<int> max_pairs[64];
    if ((rc = set_smem_attr(kern, kPairSmemBytes, attr_set))) return rc;
    int dev = 0;
    cudaGetDevice(&dev);
    int pairs = num_sms() / 2;
    if (dev < 64) {
      int known = max_pairs[dev].load(std::memory_order_acquire);
      if (known == 0) {
        // clusters that can be resident at once (GPCs may leave an SM unpaired)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = kPairSmemBytes;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
          cudaGetLastError();
          n = pairs;
        }
        max_pairs[dev].store(n, std::memory_order_release);
        known = n;
      }
      pairs = known;
    }
    const int grid_pairs = p.num_tiles < pairs ? p.num_tiles : pairs;
    LaunchScope scope(kKindGemm, stream);
    err = launch_maybe_dependent(kern, 2 * grid_pairs, kPairSmemBytes, stream, p.wait_prev != 0, tx,
                                 tw, tx2, tw2, p);
  } else {
    auto kern = lora_gemm_kernel<kWMN, kBF16, OutT>;
    static std::atomic<bool> attr_set[64];
    if ((rc = set_smem_attr(kern, kSmemBytes, attr_set))) return rc;
    const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
    LaunchScope scope(kKindGemm, stream);
    err = launch_maybe_dependent(kern, grid, kSmemBytes, stream, p.wait_prev != 0, tx, tw, tx2, tw2,
                                 p);
  }
  if (err != cudaSuccess) {
    set_error(std::string("gemm launch: ") + cudaGetErrorString(err));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

}  // namespace

int launch_gemm(const GemmArgs& a, cudaStream_t stream) {
  const bool bf16 = a.elt == Elt::kBF16;
  if (a.out_dtype == MLORA_DTYPE_F32) {
    if (a.w_mn_major)
      return bf16 ? launch_typed<true, true, float>(a, stream)
                  : launch_typed<true, false, float>(a, stream);
    return bf16 ? launch_typed<false, true, float>(a, stream)
                : launch_typed<false, false, float>(a, stream);
  }
  if (bf16) {
    return a.w_mn_major ? launch_typed<true, true, __nv_bfloat16>(a, stream)
                        : launch_typed<false, true, __nv_bfloat16>(a, stream);
  }
  return a.w_mn_major ? launch_typed<true, false, __half>(a, stream)
                      : launch_typed<false, false, __half>(a, stream);
}

}  // namespace mlora
