// Decode-size LoRA linear (M <= 16 tokens): HBM-bound on the base weight.
//
//   sT[m, j] = s * sum_k x[m, k] A[j, k]                             (lora_rank_small_kernel)
//   y[m, n]  = sum_k W[n, k] x[m, k] + sum_j B[n, j] sT[m, j]        (lora_decode_kernel)
//
// lora_decode_kernel is persistent.  Work items are (128-row block, k-split)
// pairs; per CTA:
//   warp 0      TMA producer: per stage, one [128 rows x 128 bytes] box of
//               weight rows (128-byte swizzle) and, for quantised bases, the
//               matching box of the prepared scale table [groups, rows];
//   warps 2..   tensor cores: each owns two 16-row tiles and issues
//               mma.m16n8k16 with the WEIGHTS as the A operand and the tokens
//               (staged once per item in shared memory) as B, so one token
//               fragment feeds both tiles.
// Dequantisation never multiplies per weight:
//   NF4   a 256-entry table (one copy per lane, so lookups never conflict) maps
//         a code byte to the bf16 pair (L[lo], L[hi]) of the reference's
//         4-decimal levels; the block absmax scales the fp32 sum of each quad;
//   INT4  0x4300 | q is the bf16 value 128 + q; minus (128 + zero) it is the
//         exact integer q - zero; the group scale multiplies the quad sum;
//   INT8  2^23 + q built in fp32 by a byte permute, minus (2^23 + zero), is the
//         exact q - zero, which bf16 holds exactly (|q - zero| < 256).
// Every product is therefore exact up to the bf16 rounding of the NF4 levels,
// and each scale applies once per quad in fp32: within the bf16 tolerance of
// the reference's dequantise-then-multiply order, and deterministic.
// With one k-split per row block the fragments get the rank-r term and are
// written to y directly; otherwise split partials go to a workspace and the
// last CTA of each row block sums them in split order, adds the rank-r term
// and writes y.
#include <algorithm>
#include <atomic>
#include <string>

#include "internal.h"
#include "ptx.cuh"
#include "quant.cuh"
#include "../../include/metallora_b200.h"

namespace mlora {
namespace {

constexpr int kDecRows = 128;     // output rows per work item
constexpr int kRowGroups = 4;     // MMA warps per k part, 32 rows (two 16-row tiles) each
constexpr int kBoxBytes = 128;    // inner extent of one TMA box (128-byte swizzle)
constexpr int kStageBytes = kDecRows * kBoxBytes;  // 16 KB
constexpr int kMaxTok = 16;
constexpr int kSmemPerSm = 227 * 1024;

// scheme 0 = dense bf16 weights, else QuantScheme.
template <int kScheme>
struct Dec {
  static constexpr int kBits = kScheme == 0 ? 16 : (kScheme == kINT8 ? 8 : 4);
  static constexpr int kStageK = kBoxBytes * 8 / kBits;  // k per stage: 64 / 128 / 256
  static constexpr int kQuads = kStageK / 64;            // 64-wide k quads per stage
  static constexpr int kQuadBytes = 64 * kBits / 8;      // bytes of one quad of one row
  static constexpr bool kScaled = kScheme != 0;
  static constexpr int kStages = 4;
  // NF4 pair table: 256 entries, one copy per 16 lanes (at most 2-way bank
  // conflicts), small enough for two CTAs per SM
  static constexpr int kLutCopies = 16;
  static constexpr int kLutBytes = kScheme == kNF4 ? 256 * kLutCopies * 4 : 0;
  static constexpr int kScaleSlot = 4 * kDecRows * 4;  // up to 4 groups x 128 rows x 4 bytes
  static constexpr int kScaleBytes = kScaled ? kStages * kScaleSlot : 0;
  static constexpr int kMinBlocks = 2;  // registers sized for two CTAs per SM
  // k parts: the quads of each stage are dealt round-robin to kKS groups of
  // kRowGroups MMA warps (more warps to hide the table-lookup latency of NF4);
  // the groups' accumulators are summed in order at the end of each item
  static constexpr int kKS = 1;
  static constexpr int kConsumers = kRowGroups * kKS;
  static constexpr int kThreads = 64 + 32 * kConsumers;
  static constexpr int kRedBytes = (kKS - 1) * kRowGroups * 32 * 16 * 4;
};

struct DecParams {
  const __nv_bfloat16* x;  // [M, K]
  const __nv_bfloat16* b;  // [N, r] (nullptr: no rank term)
  const float* st;         // [st_splits, M, r] partial sums of s.x.A^T
  int st_splits;
  __nv_bfloat16* y;        // [M, N]
  float* partials;         // [splits, M, N]
  uint32_t* counters;      // [row blocks]
  int M, N, K, r, group, gps;  // gps: scale-table groups per stage box
  int splits, kspan, items, row_blocks;
  long long ldy;  // row stride of y
  uint32_t* status;
};

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&a),
                             *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// The four A-fragment words of one 16-row tile for MMA step b of a quad:
// {row g: k+0,1 | row g+8: k+0,1 | row g: k+2,3 | row g+8: k+2,3}, k = 16q + 4b
// within the quad (INT4 pairs (k, k+2) and (k+1, k+3) instead; its tokens are
// staged in that order).  w0 / w1: the lane's words of rows g / g+8; z0 / z1:
// their offset words.
template <int kScheme, int kWords>
__device__ __forceinline__ void a_frags(const uint32_t (&w0)[kWords], const uint32_t (&w1)[kWords],
                                        uint32_t z0, uint32_t z1, int b, const uint32_t* lut_lane,
                                        uint32_t (&a)[4]) {
  if constexpr (kScheme == 0) {
    a[0] = w0[2 * b];
    a[2] = w0[2 * b + 1];
    a[1] = w1[2 * b];
    a[3] = w1[2 * b + 1];
  } else if constexpr (kScheme == kNF4) {
    // word b/2 holds k 8(b/2)..+7; its bytes 2(b%2), 2(b%2)+1 are k+0,1 and k+2,3
    const uint32_t s0 = (b & 1) ? 0x4442u : 0x4440u, s1 = (b & 1) ? 0x4443u : 0x4441u;
    const uint32_t u0 = w0[b >> 1], u1 = w1[b >> 1];
    constexpr int kC = Dec<kScheme>::kLutCopies;
    a[0] = lut_lane[__byte_perm(u0, 0, s0) * kC];
    a[2] = lut_lane[__byte_perm(u0, 0, s1) * kC];
    a[1] = lut_lane[__byte_perm(u1, 0, s0) * kC];
    a[3] = lut_lane[__byte_perm(u1, 0, s1) * kC];
  } else if constexpr (kScheme == kINT4) {
    const uint32_t sel = (b & 1) ? 0x4342u : 0x4140u;  // code bytes -> bits 0-7 and 16-23
    const uint32_t t0 = __byte_perm(w0[b >> 1], 0, sel), t1 = __byte_perm(w1[b >> 1], 0, sel);
    a[0] = bf16x2_sub((t0 & 0x000F000Fu) | 0x43004300u, z0);         // (k, k+2)
    a[2] = bf16x2_sub(((t0 >> 4) & 0x000F000Fu) | 0x43004300u, z0);  // (k+1, k+3)
    a[1] = bf16x2_sub((t1 & 0x000F000Fu) | 0x43004300u, z1);
    a[3] = bf16x2_sub(((t1 >> 4) & 0x000F000Fu) | 0x43004300u, z1);
  } else {  // INT8: word b holds k+0..3
    const float f0 = __uint_as_float(z0), f1 = __uint_as_float(z1);
    const uint32_t u0 = w0[b], u1 = w1[b];
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[i] = __fsub_rn(__uint_as_float(__byte_perm(u0, 0x4B000000u, 0x7440u + i)), f0);
      f[4 + i] = __fsub_rn(__uint_as_float(__byte_perm(u1, 0x4B000000u, 0x7440u + i)), f1);
    }
    a[0] = pack2<__nv_bfloat16>(f[0], f[1]);
    a[2] = pack2<__nv_bfloat16>(f[2], f[3]);
    a[1] = pack2<__nv_bfloat16>(f[4], f[5]);
    a[3] = pack2<__nv_bfloat16>(f[6], f[7]);
  }
}

// out[m] += sum_j B[n, j] sT[m, j] for one row (brow = B + n*r; sts = [M, r]
// in shared memory); the row's loads go out 8 at a time.
__device__ __forceinline__ void add_rank_term(const __nv_bfloat16* brow, const float* sts, int M,
                                              int r, float (&out)[kMaxTok]) {
  for (int j0 = 0; j0 < r; j0 += 64) {
    uint4 bv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      bv[u] = j0 + 8 * u < r ? __ldg(reinterpret_cast<const uint4*>(brow + j0 + 8 * u))
                             : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (j0 + 8 * u >= r) break;
      const __nv_bfloat162* bp = reinterpret_cast<const __nv_bfloat162*>(&bv[u]);
      float bf[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(bp[i]);
        bf[2 * i] = f.x;
        bf[2 * i + 1] = f.y;
      }
#pragma unroll
      for (int m = 0; m < kMaxTok; ++m) {
        if (m < M) {
          const float* sm = sts + m * r + j0 + 8 * u;
#pragma unroll
          for (int i = 0; i < 8; ++i) out[m] = fmaf(bf[i], sm[i], out[m]);
        }
      }
    }
  }
}

template <int kScheme, int kNT>
__global__ void __launch_bounds__(Dec<kScheme>::kThreads, Dec<kScheme>::kMinBlocks)
    lora_decode_kernel(const __grid_constant__ CUtensorMap wmap,
                       const __grid_constant__ CUtensorMap smap, const DecParams p) {
  using D = Dec<kScheme>;
  constexpr int kWords = D::kQuadBytes / 16;  // 32-bit words per lane per row per quad: 2/4/8
  extern __shared__ uint8_t smem_raw[];
  // ring (1024-byte aligned for the 128-byte swizzle) | scale slots | lut |
  // k-part partial sums | rank term per row | sT [M, r] | tokens [M, kspan + 4]
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t* scl = reinterpret_cast<const uint32_t*>(ring + D::kStages * kStageBytes);
  uint32_t* lut = reinterpret_cast<uint32_t*>(ring + D::kStages * kStageBytes + D::kScaleBytes);
  float* red = reinterpret_cast<float*>(ring + D::kStages * kStageBytes + D::kScaleBytes +
                                        D::kLutBytes);
  float* rt = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(red) + D::kRedBytes);
  float* sts = rt + kMaxTok * kDecRows;
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(sts + ((kMaxTok * p.r + 3) & ~3));
  __shared__ __align__(8) uint64_t full_bar[D::kStages];
  __shared__ __align__(8) uint64_t empty_bar[D::kStages];
  __shared__ __align__(8) uint64_t st_bar;    // sT folded into shared memory
  __shared__ __align__(8) uint64_t rt_full;   // rank term of the current item's rows ready
  __shared__ __align__(8) uint64_t rt_empty;  // ... and consumed
  __shared__ uint32_t last_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int stages_per_item = p.kspan / D::kStageK;
  const int xstride = p.kspan + 4;  // bf16 elements: rows 8 bytes off a 128-byte multiple

  if (threadIdx.x == 0) {
    for (int s = 0; s < D::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], D::kConsumers);
    }
    mbar_init(&st_bar, 1);
    mbar_init(&rt_full, 1);
    mbar_init(&rt_empty, kRowGroups);
    fence_mbarrier_init();
  }
  if constexpr (kScheme == kNF4) {
    // lut[e * kLutCopies + c] = (bf16 L[e & 15], bf16 L[e >> 4]) for every copy c
    for (int i = threadIdx.x; i < 256 * D::kLutCopies; i += blockDim.x) {
      const int e = i / D::kLutCopies;
      lut[i] = pack2<__nv_bfloat16>(kNF4Levels[e & 15], kNF4Levels[e >> 4]);
    }
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      prefetch_tmap(&wmap);
      if constexpr (D::kScaled) prefetch_tmap(&smap);
      const uint32_t stage_tx = kStageBytes + (D::kScaled ? p.gps * kDecRows * 4 : 0);
      bool ok = true;
      uint32_t it = 0;
      for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x) {
        const int rb = item % p.row_blocks, split = item / p.row_blocks;
        const int kb0 = split * p.kspan * D::kBits / 8;
        for (int sl = 0; sl < stages_per_item; ++sl) {
          const int s = it % D::kStages;
          if (!mbar_wait(&empty_bar[s], ((it / D::kStages) & 1) ^ 1, p.status, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[s], stage_tx);
          tma_load_2d(ring + s * kStageBytes, &wmap, &full_bar[s], kb0 + sl * kBoxBytes,
                      rb * kDecRows);
          if constexpr (D::kScaled)  // [gps groups x 128 rows] of the prepared scale table
            tma_load_2d(ring + D::kStages * kStageBytes + s * D::kScaleSlot, &smap, &full_bar[s],
                        rb * kDecRows, (split * p.kspan + sl * D::kStageK) / p.group);
          ++it;
        }
      }
      // drain: every issued stage has landed before this thread (and so the
      // CTA's shared memory) may go away
      for (uint32_t k = it > static_cast<uint32_t>(D::kStages) ? it - D::kStages : 0; k < it; ++k)
        mbar_wait(&full_bar[k % D::kStages], (k / D::kStages) & 1, p.status, kDevTimeoutDrain);
    }
    return;
  }
  if (warp == 1) {
    // ---------------------------------------------------------- rank warp --
    // sT from the preceding rank kernel (this grid's programmatic primary):
    // wait for it, fold its k-slices in order into shared memory; then, with
    // a single k-split, the rank term sum_j B[n, j] sT[m, j] of each item's
    // rows (4 rows per lane), concurrently with the consumers' stage loop.
    // B's rows of this CTA's first item go to L2 before the wait.
    auto prefetch_b = [&](int item) {
      if (p.b == nullptr || p.splits != 1 || item >= p.items) return;
      const int rb = item % p.row_blocks;
      const int rows = min(kDecRows, p.N - rb * kDecRows);
      const char* base = reinterpret_cast<const char*>(p.b + static_cast<long long>(rb) * kDecRows * p.r);
      for (int off = lane * 128; off < rows * p.r * 2; off += 32 * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(base + off));
    };
    prefetch_b(blockIdx.x);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (p.b != nullptr) {
      for (int i = lane; i < p.M * p.r; i += 32) {
        float v = 0.f;
        for (int s0 = 0; s0 < p.st_splits; s0 += 8) {  // loads in flight together
          float t8[8];
#pragma unroll
          for (int u = 0; u < 8; ++u)
            t8[u] = s0 + u < p.st_splits
                        ? __ldcg(p.st + static_cast<long long>(s0 + u) * p.M * p.r + i)
                        : 0.f;
#pragma unroll
          for (int u = 0; u < 8; ++u) v += t8[u];
        }
        sts[i] = v;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&st_bar);
    if (p.splits == 1) {
      uint32_t k = 0;
      for (int item = blockIdx.x; item < p.items; item += gridDim.x, ++k) {
        const int rb = item % p.row_blocks;
        prefetch_b(item + gridDim.x);
        if (!mbar_wait(&rt_empty, (k & 1) ^ 1, p.status, kDevTimeoutEmpty)) break;
        for (int rr = lane; rr < kDecRows; rr += 32) {
          float out[kMaxTok];
#pragma unroll
          for (int m = 0; m < kMaxTok; ++m) out[m] = 0.f;
          const int n = rb * kDecRows + rr;
          if (p.b != nullptr && n < p.N)
            add_rank_term(p.b + static_cast<long long>(n) * p.r, sts, p.M, p.r, out);
#pragma unroll
          for (int m = 0; m < kMaxTok; ++m)
            if (m < p.M) rt[m * kDecRows + rr] = out[m];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rt_full);
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers ----
  // Every consumer thread passes every named barrier, also after a timed-out
  // wait (then it skips the remaining waits and math), so none can be stranded.
  constexpr int kAll = 32 * D::kConsumers;  // consumer threads (named barrier 1)
  constexpr int kLead = 32 * kRowGroups;    // k part 0 threads (named barrier 2)
  const int cw = warp - 2;
  const int rg = cw % kRowGroups;           // 32-row group
  const int kp = cw / kRowGroups;           // k part
  const int ct = threadIdx.x - 64;          // k part 0: 0..127 = row within the block
  const int g = lane >> 2, q = lane & 3;
  const uint32_t* lut_lane = lut + (lane % D::kLutCopies);
  bool ok = true;
  uint32_t it = 0;
  uint32_t items_done = 0;  // this CTA's items so far (rt_full parity)

  for (int item = blockIdx.x; item < p.items; item += gridDim.x) {
    const int rb = item % p.row_blocks, split = item / p.row_blocks;
    const int k0 = split * p.kspan;
    // this item's token slice: M rows x kspan (zero beyond K); rows >= M are
    // never read.  Loads go out in batches of 8 per thread before any store.
    named_bar_sync(1, kAll);
    {
      const int chunks = p.M * (p.kspan / 8);
      for (int i0 = 0; i0 < chunks; i0 += 8 * kAll) {
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = i0 + u * kAll + ct;
          const int m = i / (p.kspan / 8), c = (i % (p.kspan / 8)) * 8;
          v[u] = make_uint4(0, 0, 0, 0);
          if (i < chunks && k0 + c < p.K)
            v[u] = __ldg(
                reinterpret_cast<const uint4*>(p.x + static_cast<long long>(m) * p.K + k0 + c));
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = i0 + u * kAll + ct;
          if (i >= chunks) break;
          const int m = i / (p.kspan / 8), c = (i % (p.kspan / 8)) * 8;
          uint4 w4 = v[u];
          if constexpr (kScheme == kINT4) {  // (k0, k2, k1, k3) within each group of four
            w4 = make_uint4(__byte_perm(v[u].x, v[u].y, 0x5410), __byte_perm(v[u].x, v[u].y, 0x7632),
                            __byte_perm(v[u].z, v[u].w, 0x5410), __byte_perm(v[u].z, v[u].w, 0x7632));
          }
          uint2* dst = reinterpret_cast<uint2*>(xs + m * xstride + c);
          dst[0] = make_uint2(w4.x, w4.y);
          dst[1] = make_uint2(w4.z, w4.w);
        }
      }
    }
    named_bar_sync(1, kAll);

    float acc[2][kNT][4];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[t][nt][c] = 0.f;

    for (int sl = 0; sl < stages_per_item; ++sl, ++it) {
      const int s = it % D::kStages;
      // warp-uniform, so the __syncwarp below always sees all 32 lanes
      ok = __all_sync(0xffffffffu,
                      ok && mbar_wait(&full_bar[s], (it / D::kStages) & 1, p.status,
                                      kDevTimeoutFull));
      if (!ok) continue;
      const uint8_t* stage = ring + s * kStageBytes;
#pragma unroll
      for (int j = 0; j < D::kQuads; ++j) {
        if (D::kKS > 1 && (sl * D::kQuads + j) % D::kKS != kp) continue;  // another k part's
        // the lane's words of rows g and g+8 of both tiles (swizzled 16-byte chunks)
        uint32_t w[2][2][kWords];
        uint2 e[2][2];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int row = rg * 32 + t * 16 + h * 8 + g;
            const uint8_t* rp = stage + row * kBoxBytes;
            if constexpr (kWords == 2) {
              const int off = j * D::kQuadBytes + 8 * q;
              const uint2 v = *reinterpret_cast<const uint2*>(
                  rp + ((((off >> 4) ^ g) << 4) | (off & 15)));
              w[t][h][0] = v.x;
              w[t][h][1] = v.y;
            } else if constexpr (kWords == 4) {
              const int chunk = (j * D::kQuadBytes >> 4) + q;
              const uint4 v = *reinterpret_cast<const uint4*>(rp + ((chunk ^ g) << 4));
              w[t][h][0] = v.x;
              w[t][h][1] = v.y;
              w[t][h][2] = v.z;
              w[t][h][3] = v.w;
            } else {
              const uint4 v0 = *reinterpret_cast<const uint4*>(rp + (((2 * q) ^ g) << 4));
              const uint4 v1 = *reinterpret_cast<const uint4*>(rp + (((2 * q + 1) ^ g) << 4));
              w[t][h][0] = v0.x;
              w[t][h][1] = v0.y;
              w[t][h][2] = v0.z;
              w[t][h][3] = v0.w;
              w[t][h][4] = v1.x;
              w[t][h][5] = v1.y;
              w[t][h][6] = v1.z;
              w[t][h][7] = v1.w;
            }
            if constexpr (D::kScaled) {
              // prepared table: NF4 absmax (fp32) or (scale, zero) fp16 pair
              const uint32_t wv = scl[s * (D::kScaleSlot / 4) + ((j * 64) / p.group) * kDecRows + row];
              if constexpr (kScheme == kNF4) {
                e[t][h] = make_uint2(wv, 0);
              } else {
                const __half2 sz = *reinterpret_cast<const __half2*>(&wv);
                const float zf = __high2float(sz);
                e[t][h].x = __float_as_uint(__low2float(sz));
                e[t][h].y = kScheme == kINT4 ? pack2<__nv_bfloat16>(128.f + zf, 128.f + zf)  // exact
                                             : __float_as_uint(8388608.f + zf);              // exact
              }
            } else {
              e[t][h] = make_uint2(0, 0);
            }
          }
        }
        float tmp[2][kNT][4];
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) tmp[t][nt][c] = 0.f;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          uint2 xb[kNT];
          const int kk = sl * D::kStageK + j * 64 + 16 * q + 4 * b;  // k within the item
#pragma unroll
          for (int nt = 0; nt < kNT; ++nt)
            xb[nt] = (nt * 8 + g < p.M)
                         ? *reinterpret_cast<const uint2*>(xs + (nt * 8 + g) * xstride + kk)
                         : make_uint2(0, 0);
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            uint32_t a[4];
            a_frags<kScheme, kWords>(w[t][0], w[t][1], e[t][0].y, e[t][1].y, b, lut_lane, a);
#pragma unroll
            for (int nt = 0; nt < kNT; ++nt) {
              if constexpr (D::kScaled)
                mma16816(tmp[t][nt], a, xb[nt].x, xb[nt].y);
              else
                mma16816(acc[t][nt], a, xb[nt].x, xb[nt].y);
            }
          }
        }
        if constexpr (D::kScaled) {
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const float s0 = __uint_as_float(e[t][0].x), s1 = __uint_as_float(e[t][1].x);
#pragma unroll
            for (int nt = 0; nt < kNT; ++nt) {
              acc[t][nt][0] = fmaf(s0, tmp[t][nt][0], acc[t][nt][0]);
              acc[t][nt][1] = fmaf(s0, tmp[t][nt][1], acc[t][nt][1]);
              acc[t][nt][2] = fmaf(s1, tmp[t][nt][2], acc[t][nt][2]);
              acc[t][nt][3] = fmaf(s1, tmp[t][nt][3], acc[t][nt][3]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[s]);
    }

    if constexpr (D::kKS > 1) {
      // k parts 1.. hand their sums to part 0, which adds them in part order
      float* mine = red + ((kp - 1) * kRowGroups + rg) * 32 * 16 + lane * 16;
      if (kp > 0) {
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) mine[(t * kNT + nt) * 4 + c] = acc[t][nt][c];
      }
      named_bar_sync(1, kAll);
      if (kp > 0) continue;
#pragma unroll
      for (int k2 = 1; k2 < D::kKS; ++k2) {
        const float* theirs = red + ((k2 - 1) * kRowGroups + rg) * 32 * 16 + lane * 16;
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[t][nt][c] += theirs[(t * kNT + nt) * 4 + c];
      }
    }
    // from here on k part 0 only (kLead threads, named barrier 2)

    if (p.splits == 1) {
      // whole k range in this item: fragments + the rank warp's per-row rank
      // term go straight to y (rows g, g+8; tokens 2q, 2q+1)
      const bool have_rt = mbar_wait(&rt_full, items_done & 1, p.status, kDevTimeoutFull);
      ++items_done;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = rg * 32 + t * 16 + h * 8 + g;
          const int n = rb * kDecRows + row;
          if (n >= p.N) continue;
#pragma unroll
          for (int nt = 0; nt < kNT; ++nt) {
            const int m0 = nt * 8 + 2 * q;
            if (m0 >= p.M) continue;
            const float r0 = have_rt ? rt[m0 * kDecRows + row] : 0.f;
            p.y[static_cast<long long>(m0) * p.ldy + n] = __float2bfloat16_rn(acc[t][nt][2 * h] + r0);
            if (m0 + 1 < p.M) {
              const float r1 = have_rt ? rt[(m0 + 1) * kDecRows + row] : 0.f;
              p.y[static_cast<long long>(m0 + 1) * p.ldy + n] =
                  __float2bfloat16_rn(acc[t][nt][2 * h + 1] + r1);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rt_empty);
      continue;
    }

    // partial tile: C rows = output rows (g, g+8), columns = tokens (2q, 2q+1)
    float* part = p.partials + static_cast<long long>(split) * p.M * p.N;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = rb * kDecRows + rg * 32 + t * 16 + h * 8 + g;
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int m = nt * 8 + 2 * q + c;
            if (m < p.M && n < p.N)
              __stcg(part + static_cast<long long>(m) * p.N + n, acc[t][nt][2 * h + c]);
          }
        }
      }
    }
    __threadfence();
    named_bar_sync(2, kLead);
    if (ct == 0) {
      // counters are zeroed by the programmatic primary (or a memset before it)
      asm volatile("griddepcontrol.wait;" ::: "memory");
      const uint32_t ticket = atomicAdd(&p.counters[rb], 1u);
      last_flag = ticket == static_cast<uint32_t>(p.splits - 1) ? 1u : 0u;
      if (last_flag) p.counters[rb] = 0;
    }
    named_bar_sync(2, kLead);
    if (last_flag == 0) continue;
    __threadfence();
    mbar_wait(&st_bar, 0, p.status, kDevTimeoutFull);  // sT folded by the rank warp
    // last CTA of this row block: one thread per output row sums the splits
    // in order and adds the rank term
    const int n = rb * kDecRows + ct;
    if (n < p.N) {
      float out[kMaxTok];
#pragma unroll
      for (int m = 0; m < kMaxTok; ++m) {
        out[m] = 0.f;
        if (m < p.M) {
          for (int s0 = 0; s0 < p.splits; s0 += 8) {  // loads in flight together
            float t8[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
              t8[u] = s0 + u < p.splits
                          ? __ldcg(p.partials + (static_cast<long long>(s0 + u) * p.M + m) * p.N + n)
                          : 0.f;
#pragma unroll
            for (int u = 0; u < 8; ++u) out[m] += t8[u];
          }
        }
      }
      if (p.b != nullptr) add_rank_term(p.b + static_cast<long long>(n) * p.r, sts, p.M, p.r, out);
#pragma unroll
      for (int m = 0; m < kMaxTok; ++m)
        if (m < p.M) p.y[static_cast<long long>(m) * p.ldy + n] = __float2bfloat16_rn(out[m]);
    }
  }
}

// Partial sums of sT[m, j] = scale * sum_k x[m, k] A[j, k] for m < M <= 16:
// CTA (j, s) covers the s-th k slice; thread t takes 8-wide chunks t, t + 256,
// ... and loads the A chunk and every token's chunk at once (one round of
// memory latency for slices up to 2048), then the CTA reduces in a fixed
// order.  It signals its dependent grid (the decode kernel) at once so that
// grid streams weights meanwhile; the decode kernel adds the slices in order.
__global__ void __launch_bounds__(256) lora_rank_small_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ a, int M, int K, int r,
    int kslice, float scale, float* __restrict__ st, uint32_t* __restrict__ counters,
    int n_counters) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // the decode kernel's split counters (it waits for this grid before its
  // first ticket, so zeroing here needs no separate memset)
  if (blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = threadIdx.x; i < n_counters; i += blockDim.x) counters[i] = 0;
  __shared__ float red[8][kMaxTok];
  const int j = blockIdx.x, split = blockIdx.y;
  const int k0 = split * kslice, k1 = min(K, k0 + kslice);
  float acc[kMaxTok];
#pragma unroll
  for (int m = 0; m < kMaxTok; ++m) acc[m] = 0.f;
  const __nv_bfloat16* ar = a + static_cast<long long>(j) * K;
  for (int k = k0 + threadIdx.x * 8; k < k1; k += 256 * 8) {
    const uint4 av = __ldg(reinterpret_cast<const uint4*>(ar + k));
    uint4 xv[kMaxTok];
#pragma unroll
    for (int m = 0; m < kMaxTok; ++m)
      xv[m] = m < M ? __ldg(reinterpret_cast<const uint4*>(x + static_cast<long long>(m) * K + k))
                    : make_uint4(0, 0, 0, 0);
    const __nv_bfloat162* ap = reinterpret_cast<const __nv_bfloat162*>(&av);
#pragma unroll
    for (int m = 0; m < kMaxTok; ++m) {
      if (m < M) {
        const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&xv[m]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 af = __bfloat1622float2(ap[i]), xf = __bfloat1622float2(xp[i]);
          acc[m] = fmaf(xf.x, af.x, acc[m]);
          acc[m] = fmaf(xf.y, af.y, acc[m]);
        }
      }
    }
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int m = 0; m < kMaxTok; ++m) {
    if (m < M) {
      float v = acc[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[w][m] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x < M) {
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) v += red[i][threadIdx.x];
    st[(static_cast<long long>(split) * M + threadIdx.x) * r + j] = v * scale;
  }
}

int bits_of(int scheme) { return scheme == 0 ? 16 : (scheme == kINT8 ? 8 : 4); }
int stage_k_of(int scheme) { return kBoxBytes * 8 / bits_of(scheme); }

// Shared memory of one CTA: fixed regions, sT [16, r], tokens [M, kspan + 4].
template <int kScheme>
size_t smem_bytes_t(int64_t M, int64_t r, int64_t kspan) {
  using D = Dec<kScheme>;
  return 1024 + static_cast<size_t>(D::kStages) * kStageBytes + D::kScaleBytes + D::kLutBytes +
         D::kRedBytes + static_cast<size_t>(kMaxTok) * kDecRows * 4 +
         static_cast<size_t>((kMaxTok * (r > 0 ? r : 1) + 3) & ~3) * 4 +
         static_cast<size_t>(M * (kspan + 4) * 2 + 15) / 16 * 16;
}

size_t smem_bytes(int scheme, int64_t M, int64_t r, int64_t kspan) {
  switch (scheme) {
    case 0: return smem_bytes_t<0>(M, r, kspan);
    case kNF4: return smem_bytes_t<kNF4>(M, r, kspan);
    case kINT4: return smem_bytes_t<kINT4>(M, r, kspan);
    default: return smem_bytes_t<kINT8>(M, r, kspan);
  }
}

template <int kScheme, int kNT>
int launch_decode_typed(const GemvArgs& a, const DecodeConfig& cfg, cudaStream_t s) {
  using D = Dec<kScheme>;
  const int64_t row_bytes = a.K * D::kBits / 8;
  CUtensorMap map;
  if (!make_tmap_2d(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.w, static_cast<uint64_t>(row_bytes),
                    static_cast<uint64_t>(a.N), static_cast<uint64_t>(row_bytes), kBoxBytes,
                    kDecRows, true))
    return MLORA_ERR_CUDA;
  const int64_t group = a.group > 0 ? a.group : 64;
  const int gps = static_cast<int>(std::max<int64_t>(1, D::kStageK / group));
  CUtensorMap smap = map;
  if constexpr (D::kScaled) {
    if (a.scales_t == nullptr) {
      set_error("decode: quantised weight without its prepared scale table");
      return MLORA_ERR_INVALID_ARG;
    }
    const int64_t G = (a.K + group - 1) / group;
    if (!make_tmap_2d(&smap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, a.scales_t,
                      static_cast<uint64_t>(a.N), static_cast<uint64_t>(G),
                      static_cast<uint64_t>(prepared_ld(a.N)) * 4, kDecRows,
                      static_cast<uint32_t>(gps), false))
      return MLORA_ERR_CUDA;
  }
  DecParams p;
  p.x = static_cast<const __nv_bfloat16*>(a.x);
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
  p.group = static_cast<int>(group);
  p.gps = gps;
  p.splits = cfg.splits;
  p.kspan = cfg.kspan;
  p.row_blocks = static_cast<int>(gemv_row_blocks(a.N));
  p.items = p.row_blocks * cfg.splits;
  p.ldy = a.ldy > 0 ? a.ldy : a.N;
  p.status = device_status_ptr();
  const size_t smem = static_cast<size_t>(cfg.smem);
  auto kern = lora_decode_kernel<kScheme, kNT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) {
    set_error(std::string("decode attribute: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(static_cast<unsigned>(cfg.ctas));
  lc.blockDim = dim3(D::kThreads);
  lc.dynamicSmemBytes = smem;
  lc.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  LaunchScope scope(kKindGemv, s);
  e = cudaLaunchKernelEx(&lc, kern, map, smap, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("decode launch: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

template <int kScheme>
int launch_decode_scheme(const GemvArgs& a, const DecodeConfig& cfg, cudaStream_t s) {
  return a.M <= 8 ? launch_decode_typed<kScheme, 1>(a, cfg, s)
                  : launch_decode_typed<kScheme, 2>(a, cfg, s);
}

}  // namespace

int64_t gemv_row_blocks(int64_t N) { return (N + kDecRows - 1) / kDecRows; }

DecodeConfig decode_config(int scheme, int64_t M, int64_t N, int64_t K, int64_t r) {
  const int sk = stage_k_of(scheme);
  const int64_t total = (K + sk - 1) / sk;  // stages over K
  const int64_t rb = gemv_row_blocks(N);
  const int sms = num_sms();
  const size_t fixed = smem_bytes(scheme, M, r, 0);  // everything but the token slice's k
  DecodeConfig best{1, static_cast<int>(total * sk), 1, static_cast<int>(fixed)};
  double best_cost = 1e30;
  for (int per_sm = 2; per_sm >= 1; --per_sm) {  // CTAs per SM (shared memory decides)
    const int64_t cap = std::min<int64_t>(227 * 1024, kSmemPerSm / per_sm - 1024);
    if (static_cast<int64_t>(fixed) + M * sk * 2 > cap) continue;
    const int64_t kspan_max = ((cap - static_cast<int64_t>(fixed)) / (M * 2) / sk) * sk;
    const int64_t slots = static_cast<int64_t>(sms) * per_sm;
    for (int64_t per = 1; per <= total; ++per) {  // stages per split
      if (per * sk > kspan_max) break;
      const int64_t splits = (total + per - 1) / per;
      if (splits > 64) continue;
      const int64_t items = rb * splits;
      const int64_t ctas = items < slots ? items : slots;
      const int64_t rounds = (items + ctas - 1) / ctas;
      // Time in units of one stage of one CTA: the per-item fixed latency
      // (token staging, first TMA, epilogue; larger with split partials), a
      // stretch when few SMs stream, the split partials' traffic in stages
      const double active = static_cast<double>(ctas < sms ? ctas : sms);
      const double stretch = std::max(1.0, 0.55 * sms / active);
      const double fixed_t = splits == 1 ? 6.0 : 12.0;
      const double part = 2.0 * splits * M * N * 4 / (kStageBytes * static_cast<double>(ctas));
      const double cost = rounds * (per * stretch + fixed_t) + part;
      if (cost < best_cost) {
        best_cost = cost;
        best = DecodeConfig{static_cast<int>(splits), static_cast<int>(per * sk),
                            static_cast<int>(ctas),
                            static_cast<int>(smem_bytes(scheme, M, r, per * sk))};
      }
    }
  }
  return best;
}

int launch_gemv(const GemvArgs& a, cudaStream_t s) {
  if (a.M > kMaxTok) {
    set_error("decode path takes at most 16 tokens");
    return MLORA_ERR_UNSUPPORTED;
  }
  const DecodeConfig cfg = decode_config(a.scheme, a.M, a.N, a.K, a.r);
  if (cfg.splits != a.splits) {
    set_error("decode: workspace planned for a different split count");
    return MLORA_ERR_INVALID_ARG;
  }
  switch (a.scheme) {
    case 0: return launch_decode_scheme<0>(a, cfg, s);
    case kNF4: return launch_decode_scheme<kNF4>(a, cfg, s);
    case kINT4: return launch_decode_scheme<kINT4>(a, cfg, s);
    case kINT8: return launch_decode_scheme<kINT8>(a, cfg, s);
    default: set_error("decode: unknown scheme"); return MLORA_ERR_INVALID_ARG;
  }
}

int rank_small_splits(int64_t K) {
  const int64_t s = (K + 2047) / 2048;  // ~2048 k per CTA
  return static_cast<int>(s < 1 ? 1 : (s > 16 ? 16 : s));
}

int launch_rank_small(const void* x, const void* a, int64_t M, int64_t K, int64_t r, float scale,
                      float* st, uint32_t* counters, int64_t n_counters, cudaStream_t s) {
  // same shared-memory carveout as the decode kernel that follows, so SMs
  // need no reconfiguration between the two (a hint, set once per device)
  static std::atomic<bool> carve_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !carve_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(lora_rank_small_kernel,
                             cudaFuncAttributePreferredSharedMemoryCarveout,
                             static_cast<int>(cudaSharedmemCarveoutMaxShared)) != cudaSuccess)
      cudaGetLastError();  // a hint only: clear the error, launch without it
    else if (dev < 64)
      carve_set[dev].store(true, std::memory_order_release);
  }
  LaunchScope scope(kKindGemv, s);
  const int splits = rank_small_splits(K);
  const int64_t kslice = ((K + splits - 1) / splits + 7) / 8 * 8;
  lora_rank_small_kernel<<<dim3(static_cast<unsigned>(r), static_cast<unsigned>(splits)), 256, 0,
                           s>>>(static_cast<const __nv_bfloat16*>(x),
                                static_cast<const __nv_bfloat16*>(a), static_cast<int>(M),
                                static_cast<int>(K), static_cast<int>(r),
                                static_cast<int>(kslice), scale, st, counters,
                                static_cast<int>(n_counters));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("rank_small launch: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

}  // namespace mlora
