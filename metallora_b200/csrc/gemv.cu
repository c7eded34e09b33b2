// Decode-size LoRA linear (M <= 16 tokens): HBM-bound on the base weight.
//
//   sT[m, j] = s * sum_k x[m, k] A[j, k]                             (lora_rank_small_kernel)
//   y[m, n]  = sum_k W[n, k] x[m, k] + sum_j B[n, j] sT[m, j]        (lora_decode_kernel)
//
// lora_decode_kernel is persistent, one CTA per SM.  The weight is cut into
// units of (128-row block, one stage of k); unit u = row_block * S + stage,
// and CTA i streams the contiguous unit range [U i / P, U (i + 1) / P) of the
// U units (stream-K), so every SM gets the same number of weight bytes to
// within one stage whatever the shape.  A CTA's range splits at row-block
// boundaries into segments:
//   whole    a complete row block: summed here and written to y;
//   publish  the part of a row block before its end (the range's last
//            segment): summed here and stored as this CTA's one fp32 partial
//            [M, 128];
//   finish   the end of a row block that began in earlier CTAs (the range's
//            first segment): their partials are added in CTA order, then
//            this CTA's own sum, and y is written.
// The kernel before this one (the rank kernel, or a fill kernel) sets every
// partial slot to kPartialEmpty, a signalling-NaN pattern that arithmetic
// never produces; a publisher stores its values over it once that kernel
// has completed, and a finisher polls the values themselves until none is
// kPartialEmpty -- the data is the handoff, with no flag round trip.
// Each CTA streams its publish segment first and its finish segment last, so
// a finisher only ever waits for lower CTAs' first segments: no cycles, and
// the summation order is fixed by the shape (bitwise repeatable).
//
// Per CTA:
//   warp 0      TMA producer: per stage one [128 rows x 128 bytes] box of
//               weight rows (128-byte swizzle), the matching box of the
//               prepared scale table [groups, rows] (quantised bases) and the
//               tokens' [x_rows x 64] boxes of x for the stage's k range
//               (128-byte swizzle; rows past M are zero-filled);
//   warps 1, 18, 19  (rank warps) wait for the rank kernel (programmatic
//               dependent launch), fold its sT partials into shared memory,
//               compute the rank term sum_j B[n, j] sT[m, j] of every row block
//               this CTA writes (mma.m16n8k16, tiles split three ways) while
//               the consumers stream, and pre-sum the partials a finish
//               segment needs;
//   warps 2..17 tensor cores: 4 row groups (32 rows, two 16-row tiles each)
//               x 4 k-groups (the stage's 64-wide k quads dealt round-robin);
//               mma.m16n8k16 with the WEIGHTS as the A operand and the tokens
//               as B, so one token fragment feeds two tiles; the k-groups'
//               sums meet in shared memory in fixed order at segment end.
//               Sixteen consumer warps (four per scheduler) keep the
//               shared-memory pipe busy: the NF4 pair table alone takes one
//               wavefront per 64 weights.
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
//
// k order inside a 64-wide quad: lane q of an MMA step b takes k
// 16q + 4 (b ^ f) .. + 3, f = q >> 1 for the 4-bit schemes (0 otherwise).
// The weights of lane q for the whole quad are then one contiguous 8-byte
// word pair, and the token fragment reads of the 32 lanes fall on distinct
// bank pairs of the swizzled x box (two wavefronts, the minimum).
#include <algorithm>
#include <atomic>
#include <string>

#include "internal.h"
#include "ptx.cuh"
#include "quant.cuh"
#include "../../include/metallora_b200.h"

namespace mlora {
namespace {

constexpr int kDecRows = 128;     // output rows per row block
constexpr int kBoxBytes = 128;    // inner extent of one weight box (128-byte swizzle)
constexpr int kStageBytes = kDecRows * kBoxBytes;  // 16 KB of weights per stage
constexpr int kMaxTok = 16;
constexpr int kRowGroups = 4;     // consumer warps per k-group, 32 rows each
constexpr int kKG = 4;            // k-groups (a power of two)
constexpr int kTiles = 2;         // 16-row MMA tiles per consumer warp
constexpr int kGroupRows = kTiles * 16;
static_assert(kRowGroups * kGroupRows == 128, "a row block is 128 rows");
static_assert((kKG & (kKG - 1)) == 0, "quads are dealt with a mask");
constexpr int kLutCopies = 32;    // NF4 pair table: one copy per lane
constexpr int kConsumers = kRowGroups * kKG;
constexpr int kRankWarps = 3;     // warp 1 and the two last warps
constexpr int kDecThreads = 32 * (2 + kConsumers + kRankWarps - 1);  // 640
constexpr int kSmemMax = 227 * 1024 - 1024;  // dynamic; the static barriers take the rest
constexpr int kMaxStages = 8;
// Fill pattern of an unpublished partial slot: a signalling NaN with a
// payload; arithmetic results are never signalling NaNs.
constexpr uint32_t kPartialEmpty = 0xFFBFFFFFu;

// scheme 0 = dense bf16 weights, else QuantScheme.
template <int kScheme>
struct Dec {
  static constexpr int kBits = kScheme == 0 ? 16 : (kScheme == kINT8 ? 8 : 4);
  static constexpr int kStageK = kBoxBytes * 8 / kBits;  // k per stage: 64 / 128 / 256
  static constexpr int kQuads = kStageK / 64;            // 64-wide k quads per stage
  static constexpr int kQuadBytes = 64 * kBits / 8;      // bytes of one quad of one row
  static constexpr int kWords = kQuadBytes / 16;         // 32-bit words per lane per row per quad
  static constexpr bool kScaled = kScheme != 0;
  static constexpr bool kFlip = kScheme == kNF4 || kScheme == kINT4;
};

struct DecParams {
  const __nv_bfloat16* b;  // [N, r] (nullptr: no rank term)
  const float* st;         // [st_splits, M, r] partial sums of s.x.A^T
  int st_splits;
  __nv_bfloat16* y;        // [M, ldy]
  long long ldy;
  float* partials;         // [ctas, M, 128]: one per CTA, set to kPartialEmpty before the launch
  int M, N, K, r, group, gps;
  int S;                   // stages per row block
  unsigned units;          // row blocks * S (units * ctas < 2^32, checked at launch)
  int stages;              // ring depth
  int x_rows;              // token rows of one x box (8 or 16)
  int x_slot, scale_slot;  // bytes per stage
  int off_x, off_scale, off_lut, off_red, off_rt, off_psum, off_rtf, off_sts;  // from the aligned base
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

__device__ __forceinline__ void st_relaxed_gpu(float* p, float v) {
  asm volatile("st.relaxed.gpu.global.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

__device__ __forceinline__ float4 ld_relaxed_gpu(const float4* p) {
  float4 v;
  asm volatile("ld.relaxed.gpu.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ bool partial_empty(const float4& v) {
  return __float_as_uint(v.x) == kPartialEmpty || __float_as_uint(v.y) == kPartialEmpty ||
         __float_as_uint(v.z) == kPartialEmpty || __float_as_uint(v.w) == kPartialEmpty;
}

// The four A-fragment words of one 16-row tile for MMA step b of a quad:
// {row g: k+0,1 | row g+8: k+0,1 | row g: k+2,3 | row g+8: k+2,3} with
// k = 16q + 4 bb, bb = b ^ f (INT4 pairs (k, k+2) and (k+1, k+3) instead; its
// token fragments are permuted to match).  w0 / w1: the lane's words of rows
// g / g+8; z0 / z1: their offset words; odd: bb & 1 for this lane.
template <int kScheme, int kWords>
__device__ __forceinline__ void a_frags(const uint32_t (&w0)[kWords], const uint32_t (&w1)[kWords],
                                        uint32_t z0, uint32_t z1, int b, bool odd,
                                        const uint32_t* lut_lane, uint32_t (&a)[4]) {
  if constexpr (kScheme == 0) {
    a[0] = w0[2 * b];
    a[2] = w0[2 * b + 1];
    a[1] = w1[2 * b];
    a[3] = w1[2 * b + 1];
  } else if constexpr (kScheme == kNF4) {
    // word b/2 holds k 8(b/2)..+7; its bytes 2(bb%2), 2(bb%2)+1 are k+0,1 and k+2,3
    const uint32_t s0 = odd ? 0x4442u : 0x4440u, s1 = odd ? 0x4443u : 0x4441u;
    const uint32_t u0 = w0[b >> 1], u1 = w1[b >> 1];
    constexpr int kC = kLutCopies;
    a[0] = lut_lane[__byte_perm(u0, 0, s0) * kC];
    a[2] = lut_lane[__byte_perm(u0, 0, s1) * kC];
    a[1] = lut_lane[__byte_perm(u1, 0, s0) * kC];
    a[3] = lut_lane[__byte_perm(u1, 0, s1) * kC];
  } else if constexpr (kScheme == kINT4) {
    const uint32_t sel = odd ? 0x4342u : 0x4140u;  // code bytes -> bits 0-7 and 16-23
    const uint32_t t0 = __byte_perm(w0[b >> 1], 0, sel), t1 = __byte_perm(w1[b >> 1], 0, sel);
    a[0] = bf16x2_sub((t0 & 0x000F000Fu) | 0x43004300u, z0);         // (k, k+2)
    a[2] = bf16x2_sub(((t0 >> 4) & 0x000F000Fu) | 0x43004300u, z0);  // (k+1, k+3)
    a[1] = bf16x2_sub((t1 & 0x000F000Fu) | 0x43004300u, z1);
    a[3] = bf16x2_sub(((t1 >> 4) & 0x000F000Fu) | 0x43004300u, z1);
  } else {  // INT8: word b holds k+0..3; (2^23 + q) - (2^23 + zero) on packed pairs
    const uint64_t zz0 = (static_cast<uint64_t>(z0) << 32) | z0;
    const uint64_t zz1 = (static_cast<uint64_t>(z1) << 32) | z1;
    const uint32_t u0 = w0[b], u1 = w1[b];
    uint64_t f[4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      f[i] = f2_sub((static_cast<uint64_t>(__byte_perm(u0, 0x4B000000u, 0x7441u + 2 * i)) << 32) |
                        __byte_perm(u0, 0x4B000000u, 0x7440u + 2 * i),
                    zz0);
      f[2 + i] = f2_sub((static_cast<uint64_t>(__byte_perm(u1, 0x4B000000u, 0x7441u + 2 * i)) << 32) |
                            __byte_perm(u1, 0x4B000000u, 0x7440u + 2 * i),
                        zz1);
    }
    a[0] = pack2<__nv_bfloat16>(f2_lo(f[0]), f2_hi(f[0]));
    a[2] = pack2<__nv_bfloat16>(f2_lo(f[1]), f2_hi(f[1]));
    a[1] = pack2<__nv_bfloat16>(f2_lo(f[2]), f2_hi(f[2]));
    a[3] = pack2<__nv_bfloat16>(f2_lo(f[3]), f2_hi(f[3]));
  }
}

// dst[m * 128 + row] = sum_j B[n, j] sT[m, j] for the 16-row tiles
// tile0, tile0 + tstep, ... of a row block (n = rb * 128 + row; rows past N
// give 0), on the tensor cores: B's rows are the A operand (fragments loaded
// from global memory, L2-resident after a prefetch) and sT, rounded to bf16 as
// the tensor-core paths' saved x.A^T is, the B operand; fp32 accumulation.
// sts = [M, r] fp32 in shared memory; r is a multiple of 8.
template <int kNT>
__device__ __forceinline__ void rank_rows(const __nv_bfloat16* b, const float* sts, int M, int N,
                                          int r, int rb, int tile0, int tstep, int lane,
                                          float* dst) {
  const int g = lane >> 2, q = lane & 3;
  for (int tile = tile0; tile < kDecRows / 16; tile += tstep) {
    const int row = tile * 16 + g;
    const int n0 = rb * kDecRows + row, n1 = n0 + 8;
    const uint32_t* b0p = reinterpret_cast<const uint32_t*>(b + static_cast<long long>(n0 < N ? n0 : 0) * r);
    const uint32_t* b1p = reinterpret_cast<const uint32_t*>(b + static_cast<long long>(n1 < N ? n1 : 0) * r);
    float c[kNT][4];
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) c[nt][e] = 0.f;
    for (int j0 = 0; j0 < r; j0 += 64) {
      // four 16-wide rank steps: all their B loads in flight, then the MMAs
      uint32_t a[4][4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int ja = j0 + 16 * jj + 2 * q, jb = ja + 8;  // rank pairs (ja, ja+1), (jb, jb+1)
        a[jj][0] = n0 < N && ja < r ? __ldg(b0p + ja / 2) : 0u;
        a[jj][1] = n1 < N && ja < r ? __ldg(b1p + ja / 2) : 0u;
        a[jj][2] = n0 < N && jb < r ? __ldg(b0p + jb / 2) : 0u;
        a[jj][3] = n1 < N && jb < r ? __ldg(b1p + jb / 2) : 0u;
      }
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int ja = j0 + 16 * jj + 2 * q, jb = ja + 8;
        if (j0 + 16 * jj >= r) break;
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt) {
          const int m = nt * 8 + g;
          const float* sm = sts + m * r;
          const uint32_t x0 = m < M && ja < r ? pack2<__nv_bfloat16>(sm[ja], sm[ja + 1]) : 0u;
          const uint32_t x1 = m < M && jb < r ? pack2<__nv_bfloat16>(sm[jb], sm[jb + 1]) : 0u;
          mma16816(c[nt], a[jj], x0, x1);
        }
      }
    }
    // C fragment: rows (row, row + 8) x tokens (nt*8 + 2q, +1)
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int m = nt * 8 + 2 * q + (e & 1);
        if (m < M) dst[m * kDecRows + row + (e >> 1) * 8] = c[nt][e];
      }
  }
}

// ------------------------------------------------------------- work split --

// 32-bit arithmetic throughout (the launch checks units * ctas < 2^32): the
// plan sits between kernel start and the first weight copy.
__device__ __forceinline__ unsigned unit_begin(unsigned units, int cta, int ctas) {
  return units * static_cast<unsigned>(cta) / static_cast<unsigned>(ctas);
}

// One CTA's segments in processing order: [publish], whole blocks, [finish].
struct DecPlan {
  bool has_pub, has_fin;
  int pub_rb, pub_s0, pub_s1;  // publish segment (ends before its block's end)
  int fin_rb, fin_s0;          // finish segment [fin_s0, S)
  int w_lo, n_whole;           // whole blocks w_lo .. w_lo + n_whole - 1
  int n_seg;
};

__device__ __forceinline__ DecPlan make_plan(const DecParams& p, int cta, int ctas) {
  DecPlan pl;
  const unsigned S = static_cast<unsigned>(p.S);
  const unsigned u0 = unit_begin(p.units, cta, ctas), u1 = unit_begin(p.units, cta + 1, ctas);
  const int ra = static_cast<int>(u0 / S), rb_last = static_cast<int>((u1 - 1) / S);
  const int sa = static_cast<int>(u0 - static_cast<unsigned>(ra) * S);
  const int eb = static_cast<int>(u1 - static_cast<unsigned>(rb_last) * S);  // end stage in last block
  pl.has_pub = pl.has_fin = false;
  pl.pub_rb = pl.pub_s0 = pl.pub_s1 = pl.fin_rb = pl.fin_s0 = 0;
  if (ra == rb_last) {
    const bool begins = sa == 0, ends = eb == p.S;
    pl.w_lo = ra;
    pl.n_whole = (begins && ends) ? 1 : 0;
    if (!ends) {
      pl.has_pub = true;
      pl.pub_rb = ra;
      pl.pub_s0 = sa;
      pl.pub_s1 = eb;
    } else if (!begins) {
      pl.has_fin = true;
      pl.fin_rb = ra;
      pl.fin_s0 = sa;
    }
  } else {
    int lo = ra + 1, hi = rb_last - 1;  // whole blocks between the ends
    if (sa == 0) {
      lo = ra;
    } else {
      pl.has_fin = true;
      pl.fin_rb = ra;
      pl.fin_s0 = sa;
    }
    if (eb == p.S) {
      hi = rb_last;
    } else {
      pl.has_pub = true;
      pl.pub_rb = rb_last;
      pl.pub_s0 = 0;
      pl.pub_s1 = eb;
    }
    pl.w_lo = lo;
    pl.n_whole = hi >= lo ? hi - lo + 1 : 0;
  }
  pl.n_seg = (pl.has_pub ? 1 : 0) + pl.n_whole + (pl.has_fin ? 1 : 0);
  return pl;
}

// kind: 0 whole, 1 publish, 2 finish
__device__ __forceinline__ void plan_segment(const DecPlan& pl, int S, int t, int& rb, int& s0,
                                             int& s1, int& kind) {
  if (pl.has_pub) {
    if (t == 0) {
      rb = pl.pub_rb;
      s0 = pl.pub_s0;
      s1 = pl.pub_s1;
      kind = 1;
      return;
    }
    --t;
  }
  if (t < pl.n_whole) {
    rb = pl.w_lo + t;
    s0 = 0;
    s1 = S;
    kind = 0;
    return;
  }
  rb = pl.fin_rb;
  s0 = pl.fin_s0;
  s1 = S;
  kind = 2;
}

// First CTA whose range holds unit u.
__device__ __forceinline__ int unit_owner(unsigned units, int ctas, unsigned u) {
  int j = static_cast<int>(u * static_cast<unsigned>(ctas) / units);
  if (j >= ctas) j = ctas - 1;
  while (j + 1 < ctas && unit_begin(units, j + 1, ctas) <= u) ++j;
  while (j > 0 && unit_begin(units, j, ctas) > u) --j;
  return j;
}

template <int kScheme, int kNT>
__global__ void __launch_bounds__(kDecThreads, 1)
    lora_decode_kernel(const __grid_constant__ CUtensorMap wmap,
                       const __grid_constant__ CUtensorMap smap,
                       const __grid_constant__ CUtensorMap xmap, const DecParams p) {
  using D = Dec<kScheme>;
  constexpr int kWords = D::kWords;
  extern __shared__ uint8_t smem_raw[];
  // weight ring (1024-byte aligned for the 128-byte swizzle) | x ring | scale
  // ring | lut | k-group sums | rank term [M, 128] | earlier partials [M, 128] |
  // the finish block's rank term [M, 128] | sT [M, r]
  uint8_t* base = align_smem<1024>(smem_raw);
  uint8_t* ring = base;
  uint8_t* xring = base + p.off_x;
  const uint8_t* sring = base + p.off_scale;
  uint32_t* lut = reinterpret_cast<uint32_t*>(base + p.off_lut);
  float* red = reinterpret_cast<float*>(base + p.off_red);
  float* rt = reinterpret_cast<float*>(base + p.off_rt);
  float* psum = reinterpret_cast<float*>(base + p.off_psum);
  float* rtf = reinterpret_cast<float*>(base + p.off_rtf);
  float* sts = reinterpret_cast<float*>(base + p.off_sts);
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
  __shared__ __align__(8) uint64_t rt_full;   // rank term (and earlier partials) of a block ready
  __shared__ __align__(8) uint64_t rt_empty;  // ... and consumed
  __shared__ __align__(8) uint64_t fin_ready; // the finish block's partials and rank term

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x, ctas = gridDim.x;
  // the CTA's plan lives in shared memory (read where needed, not held in
  // registers through the stage loops)
  __shared__ DecPlan pl_s;
  const DecPlan& pl = pl_s;

  // one stage's copies (weight box, scale box, the tokens' boxes), completing
  // on full_bar[slot]; issued by thread 0 only
  const uint32_t stage_tx = kStageBytes + (D::kScaled ? p.gps * kDecRows * 4 : 0) +
                            D::kQuads * p.x_rows * 128;
  auto issue_stage = [&](int slot, int rb, int s) {
    mbar_arrive_expect_tx(&full_bar[slot], stage_tx);
    tma_load_2d(ring + slot * kStageBytes, &wmap, &full_bar[slot], s * kBoxBytes, rb * kDecRows);
    if constexpr (D::kScaled)  // [gps groups x 128 rows] of the prepared scale table
      tma_load_2d(const_cast<uint8_t*>(sring) + slot * p.scale_slot, &smap, &full_bar[slot],
                  rb * kDecRows, (s * D::kStageK) / p.group);
#pragma unroll
    for (int j = 0; j < D::kQuads; ++j)  // the tokens' k range of this stage
      tma_load_2d(xring + slot * p.x_slot + j * p.x_rows * 128, &xmap, &full_bar[slot],
                  s * D::kStageK + 64 * j, 0);
  };

  if (threadIdx.x == 0) {
    // the descriptor fetches overlap the plan and the barrier set-up
    prefetch_tmap(&wmap);
    prefetch_tmap(&xmap);
    if constexpr (D::kScaled) prefetch_tmap(&smap);
    pl_s = make_plan(p, cta, ctas);
    // the first stage's copies leave before the rest of the set-up (every
    // CTA has at least one unit: the grid is at most the unit count)
    mbar_init(&full_bar[0], 1);
    fence_mbarrier_init();
    {
      int rb, s0, s1, kind;
      plan_segment(pl_s, p.S, 0, rb, s0, s1, kind);
      issue_stage(0, rb, s0);
    }
    for (int s = 0; s < p.stages; ++s) {
      if (s > 0) mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kConsumers);
    }
    mbar_init(&rt_full, kRankWarps);
    mbar_init(&rt_empty, kRowGroups);
    mbar_init(&fin_ready, kRankWarps);
    fence_mbarrier_init();
  }
  // set-up barrier 2: the producer arrives as soon as the mbarriers are
  // initialised and starts streaming; the other warps first build the table
  if (warp == 0) {
    // bar.arrive is warp-aligned: lanes 1..31 must not arrive for the warp
    // before lane 0 has initialised the barriers
    __syncwarp();
    named_bar_arrive(2, kDecThreads);
  } else {
    if constexpr (kScheme == kNF4) {
      // lut[e * 32 + c] = (bf16 L[e & 15], bf16 L[e >> 4]) for every lane c
      for (int i = threadIdx.x - 32; i < 256 * kLutCopies; i += blockDim.x - 32) {
        const int e = i / kLutCopies;
        lut[i] = pack2<__nv_bfloat16>(kNF4Levels[e & 15], kNF4Levels[e >> 4]);
      }
    }
    named_bar_sync(2, kDecThreads);
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      bool ok = true;
      uint32_t issued = 0;
      int slot = 0;
      uint32_t phase = 0;
      for (int t = 0; t < pl.n_seg && ok; ++t) {
        int rb, s0, s1, kind;
        plan_segment(pl, p.S, t, rb, s0, s1, kind);
        for (int s = s0; s < s1; ++s) {
          if (issued > 0) {  // the first stage left during the set-up
            if (!mbar_wait(&empty_bar[slot], phase ^ 1, p.status, kDevTimeoutEmpty)) {
              ok = false;
              break;
            }
            issue_stage(slot, rb, s);
          }
          ++issued;
          if (++slot == p.stages) {
            slot = 0;
            phase ^= 1;
          }
        }
      }
      // drain: every issued stage has landed before this thread (and so the
      // CTA's shared memory) may go away
      const uint32_t st = static_cast<uint32_t>(p.stages);
      for (uint32_t k = issued > st ? issued - st : 0; k < issued; ++k)
        mbar_wait(&full_bar[k % st], (k / st) & 1, p.status, kDevTimeoutDrain);
    }
    return;
  }
  if (warp == 1 || warp >= 2 + kConsumers) {
    // --------------------------------------------------------- rank warps --
    // three warps fold sT and pre-sum the finish block's earlier partials
    // together; the 16-row tiles of every rank term are dealt round-robin
    // over the three
    const int rw = warp == 1 ? 0 : warp - (1 + kConsumers);
    constexpr int kRankAll = 32 * kRankWarps;  // named barrier 3
    auto prefetch_rows = [&](int rb) {  // B rows of a row block this CTA writes, to L2
      if (p.b == nullptr) return;
      const int rows = min(kDecRows, p.N - rb * kDecRows);
      const char* bp = reinterpret_cast<const char*>(p.b + static_cast<long long>(rb) * kDecRows * p.r);
      for (int off = (rw * 32 + lane) * 128; off < rows * p.r * 2; off += kRankAll * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(bp + off));
    };
    auto rows_of = [&](int rb, float* dst) {  // this warp's tiles of the block
      rank_rows<kNT>(p.b, sts, p.M, p.N, p.r, rb, rw, kRankWarps, lane, dst);
    };
    if (pl.has_fin) prefetch_rows(pl.fin_rb);
    if (pl.n_whole > 0) prefetch_rows(pl.w_lo);
    // sT comes from the preceding rank kernel (this grid's programmatic
    // primary), which also set the partial slots to kPartialEmpty
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (p.b != nullptr) {
      // sT = the sum of the rank kernel's K splits, in split order
      const int n = p.M * p.r;
      if ((n & 3) == 0) {
        // four elements per load; two float4 lanes x four splits in flight
        const int n4 = n >> 2;
        const float4* st4 = reinterpret_cast<const float4*>(p.st);
        float4* sts4 = reinterpret_cast<float4*>(sts);
        for (int i0 = rw * 32 + lane; i0 < n4; i0 += 2 * kRankAll) {
          float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
          for (int s0 = 0; s0 < p.st_splits; s0 += 4) {
            float4 v[4][2];
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int i = i0 + e * kRankAll;
                v[u][e] = s0 + u < p.st_splits && i < n4
                              ? __ldcg(st4 + static_cast<long long>(s0 + u) * n4 + i)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (s0 + u < p.st_splits)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  acc[e].x += v[u][e].x;
                  acc[e].y += v[u][e].y;
                  acc[e].z += v[u][e].z;
                  acc[e].w += v[u][e].w;
                }
          }
#pragma unroll
          for (int e = 0; e < 2; ++e)
            if (i0 + e * kRankAll < n4) sts4[i0 + e * kRankAll] = acc[e];
        }
      } else {
        for (int i = rw * 32 + lane; i < n; i += kRankAll) {
          float v = 0.f;
          for (int s0 = 0; s0 < p.st_splits; s0 += 8) {  // loads in flight together
            float t8[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
              t8[u] = s0 + u < p.st_splits ? __ldcg(p.st + static_cast<long long>(s0 + u) * n + i)
                                           : 0.f;
#pragma unroll
            for (int u = 0; u < 8; ++u)
              if (s0 + u < p.st_splits) v += t8[u];
          }
          sts[i] = v;
        }
      }
      named_bar_sync(3, kRankAll);
      // the rank terms of the finish block and of the first whole block while
      // the consumers stream (the finish block is streamed last)
      if (pl.has_fin) rows_of(pl.fin_rb, rtf);
    }
    int w = 0;  // whole blocks whose rank term is staged
    if (pl.n_whole > 0) {  // the first one at once (its buffer starts free)
      if (p.b != nullptr) rows_of(pl.w_lo, rt);
      __syncwarp();
      if (lane == 0) mbar_arrive(&rt_full);
      w = 1;
    }
    if (pl.has_fin) {
      // the partials of the CTAs before this one that cover the start of the
      // finish block (their publish segments come first), summed in CTA
      // (= k) order, ready long before this CTA streams the block's end; the
      // three rank warps take every third group of 32 float4s
      const int jlo = unit_owner(p.units, ctas, static_cast<unsigned>(pl.fin_rb) * static_cast<unsigned>(p.S));
      // partials summed in publisher (= k) order, two elements x four
      // publishers of loads in flight per round; a round is reloaded until
      // none of its values is kPartialEmpty (bounded)
      bool ok = true;
      const uint64_t t0 = globaltimer_ns();
      const int n4 = p.M * kDecRows / 4;
      const float4* parts = reinterpret_cast<const float4*>(p.partials);
      float4* ps4 = reinterpret_cast<float4*>(psum);
      constexpr int kE = 2, kP = 4;
      for (int i0 = rw * 32 + lane; i0 < n4; i0 += kE * kRankAll) {
        float4 acc[kE];
#pragma unroll
        for (int u = 0; u < kE; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j0 = jlo; j0 < cta; j0 += kP) {
          float4 v[kP][kE];
          for (uint32_t spins = 1;; ++spins) {
            bool ready = true;
#pragma unroll
            for (int jj = 0; jj < kP; ++jj)
#pragma unroll
              for (int u = 0; u < kE; ++u) {
                const int i = i0 + u * kRankAll;
                v[jj][u] = j0 + jj < cta && i < n4
                               ? ld_relaxed_gpu(parts + static_cast<long long>(j0 + jj) * n4 + i)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
                ready = ready && !partial_empty(v[jj][u]);
              }
            if (ready || !ok) break;
            if ((spins & 15u) == 0 && globaltimer_ns() - t0 > MLORA_WAIT_BUDGET_NS) {
              record_status(p.status, kDevTimeoutReduce);
              ok = false;
            }
          }
#pragma unroll
          for (int jj = 0; jj < kP; ++jj) {  // in publisher order
            if (j0 + jj < cta) {
#pragma unroll
              for (int u = 0; u < kE; ++u) {
                acc[u].x += v[jj][u].x;
                acc[u].y += v[jj][u].y;
                acc[u].z += v[jj][u].z;
                acc[u].w += v[jj][u].w;
              }
            }
          }
        }
#pragma unroll
        for (int u = 0; u < kE; ++u)
          if (i0 + u * kRankAll < n4) ps4[i0 + u * kRankAll] = acc[u];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&fin_ready);
    }
    for (; w < pl.n_whole; ++w) {
      if (w + 1 < pl.n_whole) prefetch_rows(pl.w_lo + w + 1);
      if (!mbar_wait(&rt_empty, (w & 1) ^ 1, p.status, kDevTimeoutEmpty)) break;
      if (p.b != nullptr) rows_of(pl.w_lo + w, rt);
      __syncwarp();
      if (lane == 0) mbar_arrive(&rt_full);
    }
    return;
  }

  // ------------------------------------------------------------ consumers ----
  // Every consumer thread passes every named barrier, also after a timed-out
  // wait (then it skips the math), so none can be stranded.
  constexpr int kAll = 32 * kConsumers;  // named barrier 1
  const int cw = warp - 2;
  const int rg = cw % kRowGroups;        // 32-row group
  const int kg = cw / kRowGroups;        // k-group
  const int g = lane >> 2, q = lane & 3;
  const int fq = D::kFlip ? (q >> 1) : 0;
  const uint32_t* lut_lane = lut + lane;
  // a quad's scale group: group is 64, 128 or 256, so (64 j) / group = j >> gshift
  const int gshift = p.group >= 256 ? 2 : (p.group >= 128 ? 1 : 0);
  bool ok = true;
  int slot = 0;
  uint32_t phase = 0;
  uint32_t writes = 0;  // row blocks written so far (rt_full parity)

  for (int t = 0; t < pl.n_seg; ++t) {
    int rb, s0, s1, kind;
    plan_segment(pl, p.S, t, rb, s0, s1, kind);
    float acc[kTiles][kNT][4];
#pragma unroll
    for (int i = 0; i < kTiles; ++i)
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[i][nt][c] = 0.f;

    for (int s = s0; s < s1; ++s) {
      // warp-uniform, so the __syncwarp below always sees all 32 lanes
      ok = __all_sync(0xffffffffu,
                      ok && mbar_wait(&full_bar[slot], phase, p.status, kDevTimeoutFull));
      if (ok) {
        const uint8_t* stage = ring + slot * kStageBytes;
        const uint8_t* xst = xring + slot * p.x_slot;
        const uint32_t* scl = reinterpret_cast<const uint32_t*>(sring + slot * p.scale_slot);
        // this warp's quad of the stage, if any (quads are dealt round-robin
        // over the k-groups along the row block's k); one copy of the body
        const int j = (kg - s * D::kQuads) & (kKG - 1);
        if (j < D::kQuads) {
          // the lane's words of rows g and g+8 of the four tiles (swizzled 16-byte chunks)
          uint32_t w[kTiles][2][kWords];
          uint2 e[kTiles][2];
#pragma unroll
          for (int i = 0; i < kTiles; ++i) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int row = rg * kGroupRows + i * 16 + h * 8 + g;
              const uint8_t* rp = stage + row * kBoxBytes;
              if constexpr (kWords == 2) {
                const int off = j * D::kQuadBytes + 8 * q;
                const uint2 v = *reinterpret_cast<const uint2*>(
                    rp + ((((off >> 4) ^ g) << 4) | (off & 15)));
                w[i][h][0] = v.x;
                w[i][h][1] = v.y;
              } else if constexpr (kWords == 4) {
                const int chunk = (j * D::kQuadBytes >> 4) + q;
                const uint4 v = *reinterpret_cast<const uint4*>(rp + ((chunk ^ g) << 4));
                w[i][h][0] = v.x;
                w[i][h][1] = v.y;
                w[i][h][2] = v.z;
                w[i][h][3] = v.w;
              } else {
                const uint4 v0 = *reinterpret_cast<const uint4*>(rp + (((2 * q) ^ g) << 4));
                const uint4 v1 = *reinterpret_cast<const uint4*>(rp + (((2 * q + 1) ^ g) << 4));
                w[i][h][0] = v0.x;
                w[i][h][1] = v0.y;
                w[i][h][2] = v0.z;
                w[i][h][3] = v0.w;
                w[i][h][4] = v1.x;
                w[i][h][5] = v1.y;
                w[i][h][6] = v1.z;
                w[i][h][7] = v1.w;
              }
              if constexpr (D::kScaled) {
                // prepared table: NF4 absmax (fp32) or (scale, zero) fp16 pair
                const uint32_t wv = scl[(j >> gshift) * kDecRows + row];
                if constexpr (kScheme == kNF4) {
                  e[i][h] = make_uint2(wv, 0);
                } else {
                  const __half2 sz = *reinterpret_cast<const __half2*>(&wv);
                  const float zf = __high2float(sz);
                  e[i][h].x = __float_as_uint(__low2float(sz));
                  e[i][h].y = kScheme == kINT4 ? pack2<__nv_bfloat16>(128.f + zf, 128.f + zf)  // exact
                                               : __float_as_uint(8388608.f + zf);              // exact
                }
              } else {
                e[i][h] = make_uint2(0, 0);
              }
            }
          }
          float tmp[kTiles][kNT][4];
#pragma unroll
          for (int i = 0; i < kTiles; ++i)
#pragma unroll
            for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
              for (int c = 0; c < 4; ++c) tmp[i][nt][c] = 0.f;
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const int bb = b ^ fq;
            const bool odd = (bb & 1) != 0;
            uint2 xb[kNT];
#pragma unroll
            for (int nt = 0; nt < kNT; ++nt) {
              // token row nt*8 + g of quad j's x box: 8 bytes at k 16q + 4bb
              const uint8_t* xr = xst + (j * p.x_rows + nt * 8 + g) * 128;
              const int chunk = 2 * q + (bb >> 1);
              uint2 v = *reinterpret_cast<const uint2*>(xr + ((chunk ^ g) << 4) + 8 * (bb & 1));
              if constexpr (kScheme == kINT4)  // (k, k+2) and (k+1, k+3)
                v = make_uint2(__byte_perm(v.x, v.y, 0x5410), __byte_perm(v.x, v.y, 0x7632));
              xb[nt] = v;
            }
#pragma unroll
            for (int i = 0; i < kTiles; ++i) {
              uint32_t a[4];
              a_frags<kScheme, kWords>(w[i][0], w[i][1], e[i][0].y, e[i][1].y, b, odd, lut_lane,
                                       a);
#pragma unroll
              for (int nt = 0; nt < kNT; ++nt) {
                if constexpr (D::kScaled)
                  mma16816(tmp[i][nt], a, xb[nt].x, xb[nt].y);
                else
                  mma16816(acc[i][nt], a, xb[nt].x, xb[nt].y);
              }
            }
          }
          if constexpr (D::kScaled) {
#pragma unroll
            for (int i = 0; i < kTiles; ++i) {
              const float sc0 = __uint_as_float(e[i][0].x), sc1 = __uint_as_float(e[i][1].x);
#pragma unroll
              for (int nt = 0; nt < kNT; ++nt) {
                acc[i][nt][0] = fmaf(sc0, tmp[i][nt][0], acc[i][nt][0]);
                acc[i][nt][1] = fmaf(sc0, tmp[i][nt][1], acc[i][nt][1]);
                acc[i][nt][2] = fmaf(sc1, tmp[i][nt][2], acc[i][nt][2]);
                acc[i][nt][3] = fmaf(sc1, tmp[i][nt][3], acc[i][nt][3]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[slot]);
      if (++slot == p.stages) {
        slot = 0;
        phase ^= 1;
      }
    }

    // k-groups 1..3 hand their sums to k-group 0, which adds them in order
    if (kg > 0) {
#pragma unroll
      for (int i = 0; i < kTiles; ++i)
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
          for (int c = 0; c < 4; ++c)
            red[((((kg - 1) * kRowGroups + rg) * kTiles + i) * kNT + nt) * 128 + c * 32 + lane] =
                acc[i][nt][c];
    }
    named_bar_sync(1, kAll);
    if (kg == 0) {
#pragma unroll
      for (int k2 = 1; k2 < kKG; ++k2)
#pragma unroll
        for (int i = 0; i < kTiles; ++i)
#pragma unroll
          for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c)
              acc[i][nt][c] +=
                  red[((((k2 - 1) * kRowGroups + rg) * kTiles + i) * kNT + nt) * 128 + c * 32 + lane];
    }
    named_bar_sync(1, kAll);  // the sums are read: k-groups 1..3 may go on
    if (kg != 0) continue;

    // C fragment: rows (g, g+8) of each tile = output rows; columns (2q, 2q+1)
    // of each 8-token tile = tokens
    if (kind == 1) {
      // the slots hold kPartialEmpty from the preceding kernel: overwrite
      // them only once that kernel has completed
      asm volatile("griddepcontrol.wait;" ::: "memory");
      float* part = p.partials + static_cast<long long>(cta) * p.M * kDecRows;
#pragma unroll
      for (int i = 0; i < kTiles; ++i)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = rg * kGroupRows + i * 16 + h * 8 + g;
#pragma unroll
          for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const int m = nt * 8 + 2 * q + c;
              if (m < p.M) st_relaxed_gpu(part + m * kDecRows + row, acc[i][nt][2 * h + c]);
            }
        }
      continue;
    }
    // whole: the rank term from rt (cycled with the rank warp); finish: the
    // earlier CTAs' partials and the rank term from their own buffers
    const bool have = kind == 2 ? mbar_wait(&fin_ready, 0, p.status, kDevTimeoutFull)
                                : mbar_wait(&rt_full, writes & 1, p.status, kDevTimeoutFull);
    if (kind == 0) ++writes;
    const float* rterm = kind == 2 ? rtf : rt;
#pragma unroll
    for (int i = 0; i < kTiles; ++i)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = rg * kGroupRows + i * 16 + h * 8 + g;
        const int n = rb * kDecRows + row;
        if (n >= p.N) continue;
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int m = nt * 8 + 2 * q + c;
            if (m >= p.M) continue;
            float v = acc[i][nt][2 * h + c];
            if (kind == 2 && have) v = psum[m * kDecRows + row] + v;
            if (p.b != nullptr && have) v += rterm[m * kDecRows + row];
            p.y[static_cast<long long>(m) * p.ldy + n] = __float2bfloat16_rn(v);
          }
      }
    __syncwarp();
    if (lane == 0 && kind == 0) mbar_arrive(&rt_empty);
  }
}

// Partial sums of sT[m, j] = scale * sum_k x[m, k] A[j, k] for m < M <= 16,
// on the tensor cores: CTA (jt, s) computes the 16 rank columns of tile jt over
// the s-th k slice (1024 k), each of its sixteen warps one 64-wide chunk, so
// all of a slice's loads are in flight at once; mma.m16n8k16 (A's rows as the
// A operand, the tokens as B, two 8-token tiles).  Within each 64-wide k chunk, lane q of MMA step b takes k
// 16q + 4b .. + 3 (for A and B alike), so every lane loads its 16 consecutive
// k of a row with two 16-byte loads.  The warps' sums meet in shared memory
// in warp order.  Few CTAs (16 for r 64, K 4096) keep most SMs free for the
// decode kernel, its programmatic dependent, which starts at once, streams
// weights meanwhile and adds the slices in order.
constexpr int kRankSmallWarps = 16;
constexpr int kRankThreads = 32 * kRankSmallWarps;

__global__ void __launch_bounds__(kRankThreads) lora_rank_small_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ a, int M, int K, int r,
    int kslice, float scale, float* __restrict__ st, float4* __restrict__ partials,
    int n_partials4) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // the decode kernel's partial slots to kPartialEmpty (it overwrites them
  // only after this grid has completed)
  {
    const float e = __uint_as_float(kPartialEmpty);
    const int nb = gridDim.x * gridDim.y, b = blockIdx.y * gridDim.x + blockIdx.x;
    for (int i = b * kRankThreads + threadIdx.x; i < n_partials4; i += nb * kRankThreads)
      partials[i] = make_float4(e, e, e, e);
  }
  __shared__ float red[kRankSmallWarps][16][16];  // [warp][j][m]
  const int jt = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int k0 = split * kslice, k1 = min(K, k0 + kslice);
  const int wk = (kslice / kRankSmallWarps + 63) / 64 * 64;
  const int wk0 = k0 + warp * wk, wk1 = min(k1, wk0 + wk);
  const int j0 = jt * 16 + g, j1 = j0 + 8;
  const __nv_bfloat16* a0 = j0 < r ? a + static_cast<long long>(j0) * K : nullptr;
  const __nv_bfloat16* a1 = j1 < r ? a + static_cast<long long>(j1) * K : nullptr;
  const __nv_bfloat16* x0 = g < M ? x + static_cast<long long>(g) * K : nullptr;
  const __nv_bfloat16* x1 = g + 8 < M ? x + static_cast<long long>(g + 8) * K : nullptr;
  float c[2][4];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) c[t][e] = 0.f;
  auto ld16 = [&](const __nv_bfloat16* row, int k, uint4 (&v)[2]) {
    // this lane's 16 k of a row (zero past the slice or for an absent row)
    if (row != nullptr && k + 16 <= wk1) {
      v[0] = __ldg(reinterpret_cast<const uint4*>(row + k));
      v[1] = __ldg(reinterpret_cast<const uint4*>(row + k + 8));
    } else {
      v[0] = v[1] = make_uint4(0, 0, 0, 0);
    }
  };
  for (int kc = wk0; kc < wk1; kc += 64) {
    const int k = kc + 16 * q;
    uint4 va0[2], va1[2], vx0[2], vx1[2];
    ld16(a0, k, va0);
    ld16(a1, k, va1);
    ld16(x0, k, vx0);
    ld16(x1, k, vx1);
    const uint32_t* pa0 = reinterpret_cast<const uint32_t*>(va0);
    const uint32_t* pa1 = reinterpret_cast<const uint32_t*>(va1);
    const uint32_t* px0 = reinterpret_cast<const uint32_t*>(vx0);
    const uint32_t* px1 = reinterpret_cast<const uint32_t*>(vx1);
#pragma unroll
    for (int s = 0; s < 4; ++s) {  // MMA step s: k + 4s .. + 3 (words 2s, 2s + 1)
      const uint32_t af[4] = {pa0[2 * s], pa1[2 * s], pa0[2 * s + 1], pa1[2 * s + 1]};
      mma16816(c[0], af, px0[2 * s], px0[2 * s + 1]);
      mma16816(c[1], af, px1[2 * s], px1[2 * s + 1]);
    }
  }
  // C fragment: rows (g, g + 8) = rank columns j, columns (2q, 2q + 1) of each
  // 8-token tile = tokens
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      red[warp][g + 8 * (e >> 1)][t * 8 + 2 * q + (e & 1)] = c[t][e];
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += kRankThreads) {
    const int jj = i >> 4, m = i & 15;
    const int j = jt * 16 + jj;
    if (j < r && m < M) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kRankSmallWarps; ++w) v += red[w][jj][m];
      st[(static_cast<long long>(split) * M + m) * r + j] = v * scale;
    }
  }
}

// Sets the decode kernel's partial slots to kPartialEmpty when no rank
// kernel precedes it (plain weights, no LoRA term), and lets the decode
// kernel start at once as its programmatic dependent.
__global__ void __launch_bounds__(256) lora_partials_fill_kernel(float4* __restrict__ partials,
                                                                 int n4) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const float e = __uint_as_float(kPartialEmpty);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x)
    partials[i] = make_float4(e, e, e, e);
}

int bits_of(int scheme) { return scheme == 0 ? 16 : (scheme == kINT8 ? 8 : 4); }
int stage_k_of(int scheme) { return kBoxBytes * 8 / bits_of(scheme); }
int quads_of(int scheme) { return stage_k_of(scheme) / 64; }
int x_rows_of(int64_t M) { return M <= 8 ? 8 : 16; }
int gps_of(int scheme, int64_t group) {
  return scheme == 0 ? 1 : static_cast<int>(std::max<int64_t>(1, stage_k_of(scheme) / group));
}

// Shared-memory layout of one CTA (offsets from the 1024-byte aligned base).
struct DecLayout {
  int x_slot, scale_slot;
  int off_x, off_scale, off_lut, off_red, off_rt, off_psum, off_rtf, off_sts;
  int bytes;  // including the alignment slack
};

DecLayout dec_layout(int scheme, int64_t M, int64_t r, int64_t group, int stages) {
  DecLayout L;
  const int xr = x_rows_of(M), kNT = xr / 8;
  L.x_slot = quads_of(scheme) * xr * 128;
  L.scale_slot = scheme == 0 ? 0 : gps_of(scheme, group) * kDecRows * 4;
  L.off_x = stages * kStageBytes;
  L.off_scale = L.off_x + stages * L.x_slot;
  L.off_lut = L.off_scale + stages * L.scale_slot;
  const int lut = scheme == kNF4 ? 256 * kLutCopies * 4 : 0;
  L.off_red = L.off_lut + lut;
  const int red = (kKG - 1) * kRowGroups * kTiles * kNT * 128 * 4;
  L.off_rt = L.off_red + red;
  const int tok = static_cast<int>(M) * kDecRows * 4;
  L.off_psum = L.off_rt + tok;
  L.off_rtf = L.off_psum + tok;
  L.off_sts = L.off_rtf + tok;
  L.bytes = 1024 + L.off_sts + static_cast<int>((M * (r > 0 ? r : 1) * 4 + 15) / 16 * 16);
  return L;
}

template <int kScheme, int kNT>
int launch_decode_typed(const GemvArgs& a, const DecodeConfig& cfg, cudaStream_t s) {
  using D = Dec<kScheme>;
  const int64_t row_bytes = a.K * D::kBits / 8;
  CUtensorMap wmap, xmap;
  if (!make_tmap_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.w, static_cast<uint64_t>(row_bytes),
                    static_cast<uint64_t>(a.N), static_cast<uint64_t>(row_bytes), kBoxBytes,
                    kDecRows, true))
    return MLORA_ERR_CUDA;
  const int xr = x_rows_of(a.M);
  if (!make_tmap_2d_16b(&xmap, a.x, static_cast<uint64_t>(a.K), static_cast<uint64_t>(a.M),
                        static_cast<uint64_t>(a.K), 64, static_cast<uint32_t>(xr)))
    return MLORA_ERR_CUDA;
  const int64_t group = a.group > 0 ? a.group : 64;
  const int gps = gps_of(kScheme, group);
  CUtensorMap smap = wmap;
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
  const DecLayout L = dec_layout(kScheme, a.M, a.r, group, cfg.stages);
  DecParams p;
  p.b = static_cast<const __nv_bfloat16*>(a.b);
  p.st = a.st;
  p.st_splits = a.b != nullptr ? rank_small_splits(a.K) : 0;
  p.r = static_cast<int>(a.r);
  p.y = static_cast<__nv_bfloat16*>(a.y);
  p.ldy = a.ldy > 0 ? a.ldy : a.N;
  p.partials = a.partials;
  p.M = static_cast<int>(a.M);
  p.N = static_cast<int>(a.N);
  p.K = static_cast<int>(a.K);
  p.group = static_cast<int>(group);
  p.gps = gps;
  p.S = static_cast<int>((a.K + D::kStageK - 1) / D::kStageK);
  const int64_t units = gemv_row_blocks(a.N) * p.S;
  if (units * cfg.ctas >= (int64_t(1) << 32)) {
    set_error("decode: weight too large for the 32-bit work split");
    return MLORA_ERR_UNSUPPORTED;
  }
  p.units = static_cast<unsigned>(units);
  p.stages = cfg.stages;
  p.x_rows = xr;
  p.x_slot = L.x_slot;
  p.scale_slot = L.scale_slot;
  p.off_x = L.off_x;
  p.off_scale = L.off_scale;
  p.off_lut = L.off_lut;
  p.off_red = L.off_red;
  p.off_rt = L.off_rt;
  p.off_psum = L.off_psum;
  p.off_rtf = L.off_rtf;
  p.off_sts = L.off_sts;
  p.status = device_status_ptr();
  auto kern = lora_decode_kernel<kScheme, kNT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(cfg.smem));
  if (e != cudaSuccess) {
    set_error(std::string("decode attribute: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(static_cast<unsigned>(cfg.ctas));
  lc.blockDim = dim3(kDecThreads);
  lc.dynamicSmemBytes = static_cast<size_t>(cfg.smem);
  lc.stream = s;
  // a programmatic dependent of the rank (or flag-zeroing) kernel that
  // precedes it, which writes nothing this kernel reads before
  // griddepcontrol.wait; x and the weights were complete before that kernel
  // started
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = a.pdl ? 1 : 0;
  LaunchScope scope(kKindGemv, s);
  e = cudaLaunchKernelEx(&lc, kern, wmap, smap, xmap, p);
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

DecodeConfig decode_config(int scheme, int64_t M, int64_t N, int64_t K, int64_t r, int64_t group) {
  const int sk = stage_k_of(scheme);
  const int64_t S = (K + sk - 1) / sk;
  const int64_t units = gemv_row_blocks(N) * S;
  // With a LoRA term the small rank kernel runs first, one CTA per SM, and a
  // decode CTA cannot share an SM with it: decode CTAs placed there start only
  // when it ends and finish last.  Leaving those SMs to the rank kernel makes
  // every decode CTA start at once, at the price of fewer SMs streaming.
  // Measured (same box): worth it for 16 tokens (NF4 18.7 -> 17.6 us, INT8
  // 27.3 -> 23.2 us, INT4 16.9 -> 14.3 us) and for a rank kernel of at most 8
  // CTAs at one token (INT4/INT8 r 16: -0.15 to -0.35 us); not for NF4 r 64
  // at one token (16 SMs reserved: 13.65 -> 14.02 us).
  const int64_t rank_ctas = r > 0 ? (r + 15) / 16 * rank_small_splits(K) : 0;
  const int64_t reserve = rank_ctas > 0 && (M > 8 || rank_ctas <= 8)
                              ? std::min<int64_t>(rank_ctas, num_sms() / 4) : 0;
  const int64_t ctas = std::min<int64_t>(num_sms() - reserve, units);
  const int64_t g = group > 0 ? group : 64;
  int stages = kMaxStages;
  while (stages > 2 && dec_layout(scheme, M, r, g, stages).bytes > kSmemMax) --stages;
  DecodeConfig c;
  c.ctas = static_cast<int>(ctas);
  c.stages = stages;
  c.smem = dec_layout(scheme, M, r, g, stages).bytes;
  // some row block is shared between CTAs (then the partial slots are used)
  c.split_blocks = false;
  for (int64_t j = 1; j < ctas && !c.split_blocks; ++j)
    if ((units * j / ctas) % S != 0) c.split_blocks = true;
  return c;
}

int launch_gemv(const GemvArgs& a, cudaStream_t s) {
  if (a.M > kMaxTok) {
    set_error("decode path takes at most 16 tokens");
    return MLORA_ERR_UNSUPPORTED;
  }
  const DecodeConfig cfg = decode_config(a.scheme, a.M, a.N, a.K, a.r, a.group);
  if (cfg.smem > kSmemMax) {
    set_error("decode: shared memory for rank " + std::to_string(a.r) + " exceeds the limit");
    return MLORA_ERR_UNSUPPORTED;
  }
  if (cfg.split_blocks && a.partials == nullptr) {
    set_error("decode: workspace without partials for a split row block");
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

int launch_partials_fill(float* partials, int64_t n, cudaStream_t s) {
  LaunchScope scope(kKindGemv, s);
  const int64_t n4 = n / 4;
  const int blocks = static_cast<int>(std::min<int64_t>(32, (n4 + 255) / 256));
  lora_partials_fill_kernel<<<blocks > 0 ? blocks : 1, 256, 0, s>>>(
      reinterpret_cast<float4*>(partials), static_cast<int>(n4));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("partials_fill launch: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

int rank_small_splits(int64_t K) {
  const int64_t s = (K + 1023) / 1024;  // ~1024 k per CTA
  return static_cast<int>(s < 1 ? 1 : (s > 16 ? 16 : s));
}

int launch_rank_small(const void* x, const void* a, int64_t M, int64_t K, int64_t r, float scale,
                      float* st, float* partials, int64_t n_partials, cudaStream_t s) {
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
  const int64_t kslice = ((K + splits - 1) / splits + 63) / 64 * 64;
  lora_rank_small_kernel<<<dim3(static_cast<unsigned>((r + 15) / 16), static_cast<unsigned>(splits)), kRankThreads, 0,
                           s>>>(static_cast<const __nv_bfloat16*>(x),
                                static_cast<const __nv_bfloat16*>(a), static_cast<int>(M),
                                static_cast<int>(K), static_cast<int>(r),
                                static_cast<int>(kslice), scale, st,
                                reinterpret_cast<float4*>(partials),
                                static_cast<int>(n_partials / 4));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("rank_small launch: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

}  // namespace mlora
