// Skinny tcgen05 kernels of the LoRA path (N = R_PAD <= 256 output columns):
//
//  rank projection   out[m, j] = s * sum_k X[m, k] . L[j, k]
//      forward : X = x,  L = A      -> s.x.A^T   (lora_train.metal:66 caches the same Ax)
//      backward: X = dy, L = B^T    -> s.dy.B    (ops.py:152 "bt_grad")
//  weight gradient   out[p, j] = sum_m Big[m, p] . ST[j, m]
//      dB = dy^T . (s x A^T)        (ops.py:148-149)
//      dA = (s dy B)^T . x          (ops.py:152-153), stored transposed as [r, K]
//
// Both stream one large operand once from HBM, so they are bandwidth-bound:
// each CTA keeps a deep TMA ring and several CTAs share an SM.  Work is split
// along the reduction dimension across CTAs; partial sums (fp32) go to a
// workspace and the last CTA of each output tile -- found with a counter --
// adds them in fixed split order, so results are bitwise reproducible.
//
// Warp roles: warp 0 TMA producer, warp 1 TMEM owner + UMMA issuer (M = 128,
// N = R, K = 16), warps 2-5 epilogue (one accumulator row per thread).
#include <type_traits>

#include "internal.h"
#include "ptx.cuh"
#include "../../include/metallora_b200.h"

namespace mlora {
namespace {

constexpr int kThreads = 192;
constexpr int kBK = 64;
constexpr uint32_t kBigTileBytes = 128 * kBK * 2;  // 16 KB: [128 x 64] 16-bit
constexpr uint32_t kMNBoxBytes = 64 * kBK * 2;     // 8 KB
constexpr uint32_t kSmemBudget = 100 * 1024;       // two CTAs per SM

__host__ __device__ constexpr uint32_t small_tile_bytes(int R) { return R * 128u; }
__host__ __device__ constexpr uint32_t stage_bytes(int R) {
  return kBigTileBytes + small_tile_bytes(R);
}
__host__ __device__ constexpr int num_stages(int R) {
  return static_cast<int>(kSmemBudget / stage_bytes(R)) > 8
             ? 8
             : static_cast<int>(kSmemBudget / stage_bytes(R));
}
__host__ __device__ constexpr uint32_t tmem_cols(int R) {
  return R <= 32 ? 32u : (R <= 64 ? 64u : (R <= 128 ? 128u : 256u));
}
constexpr size_t smem_bytes(int R) { return 1024 + num_stages(R) * stage_bytes(R) + 256; }

struct SplitWork {
  int tile;    // output tile (128 rows of out)
  int split;   // reduction split index
  int kb_begin, kb_end;
};

__device__ __forceinline__ SplitWork split_work(int tile, int split, int splits, int num_kb) {
  SplitWork w;
  w.tile = tile;
  w.split = split;
  const int per = (num_kb + splits - 1) / splits;
  w.kb_begin = split * per;
  w.kb_end = min(num_kb, w.kb_begin + per);
  return w;
}

// Common pipeline: produces TMEM acc [128 x R] = sum over k-blocks of
// A-tile (128 rows) x B-tile (R rows).  kAMN selects an MN-major A operand built
// from two [64 x 64] boxes (weight gradient) instead of a K-major [128 x 64] box.
template <int R, bool kAMN, bool kBF16>
__device__ __forceinline__ void run_pipeline(uint8_t* smem, uint64_t* full_bar, uint64_t* empty_bar,
                                             uint64_t* done_bar, uint32_t tmem_acc,
                                             const CUtensorMap* tm_a, const CUtensorMap* tm_b,
                                             int a_row0, int kb_begin, int kb_end,
                                             uint32_t* status) {
  constexpr int S = num_stages(R);
  const uint32_t warp = warp_id();
  if (warp == 0) {
    if (elect_one()) {
      uint32_t stage = 0, phase = 0;
      bool armed[S];
      uint32_t armed_parity[S];
      for (int s = 0; s < S; ++s) armed[s] = false, armed_parity[s] = 0;
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, status, kDevTimeoutEmpty)) break;
        uint8_t* sa = smem + stage * stage_bytes(R);
        uint8_t* sb = sa + kBigTileBytes;
        mbar_arrive_expect_tx(&full_bar[stage], stage_bytes(R));
        armed[stage] = true;
        armed_parity[stage] = phase;
        const int k0 = kb * kBK;
        if constexpr (kAMN) {
          tma_load_2d(sa, tm_a, &full_bar[stage], a_row0, k0);
          tma_load_2d(sa + kMNBoxBytes, tm_a, &full_bar[stage], a_row0 + 64, k0);
        } else {
          tma_load_2d(sa, tm_a, &full_bar[stage], k0, a_row0);
        }
        tma_load_2d(sb, tm_b, &full_bar[stage], k0, 0);
        if (++stage == S) stage = 0, phase ^= 1u;
      }
      for (int s = 0; s < S; ++s)
        if (armed[s]) mbar_wait(&full_bar[s], armed_parity[s], status, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_f16(128, R, kAMN, false, kBF16);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, status, kDevTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * stage_bytes(R));
        const uint32_t sb = sa + kBigTileBytes;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint64_t ad;
          if constexpr (kAMN)
            ad = desc_mnmajor_sw128(sa, k, kMNBoxBytes);
          else
            ad = desc_kmajor_sw128(sa, k);
          umma_f16(tmem_acc, ad, desc_kmajor_sw128(sb, k), idesc,
                   (kb != kb_begin || k != 0) ? 1u : 0u);
        }
        umma_commit(&empty_bar[stage]);
        if (++stage == S) stage = 0, phase ^= 1u;
      }
      (void)ok;
      // Signals the epilogue (and guarantees no UMMA is in flight at exit).
      umma_commit(done_bar);
    }
  }
}

// Loads this thread's accumulator row (R fp32 columns) from TMEM into `acc`.
template <int R>
__device__ __forceinline__ void load_acc_row(uint32_t taddr_row, float (&acc)[R]) {
#pragma unroll
  for (int c = 0; c < R / 16; ++c) {
    uint32_t r[16];
    tmem_ld_32x32b_x16(taddr_row + c * 16, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[c * 16 + i] = __uint_as_float(r[i]);
  }
}

// Deterministic split reduction.  Every epilogue thread owns one row of the
// [128 x R] tile.  Returns true in the CTA that must write the final result,
// with `acc` holding the sum over splits in order 0..splits-1.
template <int R>
__device__ __forceinline__ bool split_reduce(float (&acc)[R], float* partials, uint32_t* counters,
                                             int tile, int split, int splits, long long row,
                                             long long rows_total, uint32_t* flag_smem) {
  if (splits == 1) return true;
  const bool valid = row < rows_total;
  if (valid) {
    float4* dst = reinterpret_cast<float4*>(partials + (static_cast<long long>(split) * rows_total + row) * R);
#pragma unroll
    for (int i = 0; i < R / 4; ++i)
      __stcg(dst + i, make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]));
  }
  __threadfence();
  named_bar_sync(1, 128);
  if (threadIdx.x == 64) {
    const uint32_t ticket = atomicAdd(&counters[tile], 1u);
    const bool last = ticket == static_cast<uint32_t>(splits - 1);
    if (last) counters[tile] = 0;  // ready for the next launch
    *flag_smem = last ? 1u : 0u;
  }
  named_bar_sync(1, 128);
  if (*flag_smem == 0) return false;
  __threadfence();
  if (valid) {
#pragma unroll
    for (int i = 0; i < R; ++i) acc[i] = 0.f;
    // splits in order, four splits' loads in flight together
    for (int s0 = 0; s0 < splits; s0 += 4) {
#pragma unroll
      for (int i = 0; i < R / 4; ++i) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          v[u] = s0 + u < splits
                     ? __ldcg(reinterpret_cast<const float4*>(
                                  partials + (static_cast<long long>(s0 + u) * rows_total + row) * R) +
                              i)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          acc[4 * i] += v[u].x;
          acc[4 * i + 1] += v[u].y;
          acc[4 * i + 2] += v[u].z;
          acc[4 * i + 3] += v[u].w;
        }
      }
    }
  }
  return true;
}

struct RankParams {
  long long M;
  int r, num_kb, splits;
  float scale;
  void* out_rows;
  long long ld_rows;
  void* out_t;
  long long ld_t;
  int split_out;
  uint32_t split_pattern;
  float* partials;
  uint32_t* counters;
  uint32_t* status;
  const int32_t* row_group;  // optional: keep only columns [g*group_cols, (g+1)*group_cols)
  int group_cols;
};

template <int R, bool kBF16>
__global__ void __launch_bounds__(kThreads, 2)
    rank_proj_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_l,
                     const RankParams p) {
  using T = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
  constexpr int S = num_stages(R);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S * stage_bytes(R));
  uint64_t* empty_bar = full_bar + S;
  uint64_t* done_bar = empty_bar + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  uint32_t* flag = tmem_slot + 1;

  const uint32_t warp = warp_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&full_bar[s], 1), mbar_init(&empty_bar[s], 1);
    mbar_init(done_bar, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols(R));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int tile = blockIdx.x;
  const SplitWork w = split_work(tile, blockIdx.y, p.splits, p.num_kb);
  const bool has_work = w.kb_begin < w.kb_end;
  if (has_work) {
    run_pipeline<R, false, kBF16>(smem, full_bar, empty_bar, done_bar, tmem, &tm_x, &tm_l,
                                  tile * 128, w.kb_begin, w.kb_end, p.status);
  }
  if (warp >= 2) {
    const uint32_t quarter = warp & 3u;
    const long long row = static_cast<long long>(tile) * 128 + quarter * 32 + lane_id();
    float acc[R];
    bool ok = true;
    if (has_work) {
      ok = mbar_wait(done_bar, 0, p.status, kDevTimeoutAccFull);
      tc_fence_after();
      if (ok) load_acc_row<R>(tmem + ((quarter * 32u) << 16), acc);
    } else {
#pragma unroll
      for (int i = 0; i < R; ++i) acc[i] = 0.f;
    }
    if (!ok) {
#pragma unroll
      for (int i = 0; i < R; ++i) acc[i] = 0.f;
    }
    const bool final_cta =
        split_reduce<R>(acc, p.partials, p.counters, tile, w.split, p.splits, row, p.M, flag);
    if (final_cta && row < p.M && p.split_out) {
      // fp32 path: bf16 hi/lo parts of the scaled value (bf16 instantiation only)
#pragma unroll
      for (int i = 0; i < R; ++i) acc[i] *= p.scale;
      if (p.out_rows != nullptr) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out_rows) + row * p.ld_rows;
        for (int s = 0; s < 3; ++s) {
          const bool lo = (p.split_pattern >> s) & 1u;
#pragma unroll
          for (int i = 0; i < R / 2; ++i) {
            const float a0 = acc[2 * i], a1 = acc[2 * i + 1];
            const float h0 = __bfloat162float(__float2bfloat16_rn(a0));
            const float h1 = __bfloat162float(__float2bfloat16_rn(a1));
            *reinterpret_cast<uint32_t*>(dst + s * R + 2 * i) =
                lo ? pack2<__nv_bfloat16>(a0 - h0, a1 - h1) : pack2<__nv_bfloat16>(a0, a1);
          }
        }
        for (long long j = 3 * R; j < p.ld_rows; j += 8)
          *reinterpret_cast<uint4*>(dst + j) = make_uint4(0, 0, 0, 0);
      }
      if (p.out_t != nullptr) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out_t);
        for (int s = 0; s < 3; ++s) {
          const bool lo = (p.split_pattern >> s) & 1u;
#pragma unroll
          for (int j = 0; j < R; ++j) {
            const __nv_bfloat16 h = __float2bfloat16_rn(acc[j]);
            dst[static_cast<long long>(j) * p.ld_t + s * p.M + row] =
                lo ? __float2bfloat16_rn(acc[j] - __bfloat162float(h)) : h;
          }
        }
      }
    } else if (final_cta && row < p.M) {
      if (p.row_group != nullptr) {
        // stacked adapters: the row keeps only its own adapter's columns (an
        // id outside [0, R / group_cols) keeps none)
        const int g = p.row_group[row];
#pragma unroll
        for (int j = 0; j < R; ++j)
          if (j / p.group_cols != g) acc[j] = 0.f;
      }
      if (p.out_rows != nullptr) {
        T* dst = reinterpret_cast<T*>(p.out_rows) + row * p.ld_rows;
#pragma unroll
        for (int i = 0; i < R / 8; ++i) {
          uint4 v;
          v.x = pack2<T>(acc[8 * i] * p.scale, acc[8 * i + 1] * p.scale);
          v.y = pack2<T>(acc[8 * i + 2] * p.scale, acc[8 * i + 3] * p.scale);
          v.z = pack2<T>(acc[8 * i + 4] * p.scale, acc[8 * i + 5] * p.scale);
          v.w = pack2<T>(acc[8 * i + 6] * p.scale, acc[8 * i + 7] * p.scale);
          reinterpret_cast<uint4*>(dst)[i] = v;
        }
        for (long long j = R; j < p.ld_rows; j += 8)
          *reinterpret_cast<uint4*>(dst + j) = make_uint4(0, 0, 0, 0);
      }
      if (p.out_t != nullptr) {
        T* dst = reinterpret_cast<T*>(p.out_t);
#pragma unroll
        for (int j = 0; j < R; ++j) {
          if constexpr (kBF16)
            dst[static_cast<long long>(j) * p.ld_t + row] = __float2bfloat16_rn(acc[j] * p.scale);
          else
            dst[static_cast<long long>(j) * p.ld_t + row] = __float2half_rn(acc[j] * p.scale);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols(R));
  }
}

struct WgradProblem {
  long long M, P;
  int r, num_kb, splits, tiles;
  float* out;
  long long ldo;
  int transposed;
  int accumulate;
  float clip;
  float* partials;
  uint32_t* counters;
};

struct WgradParams {
  WgradProblem prob[2];
  int nprobs;
  int ctas0;  // CTAs of problem 0 (= tiles * splits)
  uint32_t* status;
};

template <int R, bool kBF16>
__global__ void __launch_bounds__(kThreads, 2)
    wgrad_kernel(const __grid_constant__ CUtensorMap tm_big0, const __grid_constant__ CUtensorMap tm_st0,
                 const __grid_constant__ CUtensorMap tm_big1, const __grid_constant__ CUtensorMap tm_st1,
                 const WgradParams p) {
  constexpr int S = num_stages(R);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S * stage_bytes(R));
  uint64_t* empty_bar = full_bar + S;
  uint64_t* done_bar = empty_bar + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  uint32_t* flag = tmem_slot + 1;

  const uint32_t warp = warp_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&full_bar[s], 1), mbar_init(&empty_bar[s], 1);
    mbar_init(done_bar, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols(R));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int which = (static_cast<int>(blockIdx.x) < p.ctas0) ? 0 : 1;
  const WgradProblem& q = p.prob[which];
  const int local = static_cast<int>(blockIdx.x) - (which ? p.ctas0 : 0);
  const int tile = local % q.tiles;
  const SplitWork w = split_work(tile, local / q.tiles, q.splits, q.num_kb);
  const bool has_work = w.kb_begin < w.kb_end;
  if (has_work) {
    run_pipeline<R, true, kBF16>(smem, full_bar, empty_bar, done_bar, tmem,
                                 which ? &tm_big1 : &tm_big0, which ? &tm_st1 : &tm_st0,
                                 tile * 128, w.kb_begin, w.kb_end, p.status);
  }
  if (warp >= 2) {
    const uint32_t quarter = warp & 3u;
    const long long prow = static_cast<long long>(tile) * 128 + quarter * 32 + lane_id();
    float acc[R];
    bool ok = true;
    if (has_work) {
      ok = mbar_wait(done_bar, 0, p.status, kDevTimeoutAccFull);
      tc_fence_after();
      if (ok) load_acc_row<R>(tmem + ((quarter * 32u) << 16), acc);
    }
    if (!has_work || !ok) {
#pragma unroll
      for (int i = 0; i < R; ++i) acc[i] = 0.f;
    }
    if (split_reduce<R>(acc, q.partials, q.counters, tile, w.split, q.splits, prow, q.P, flag) &&
        prow < q.P) {
      const bool clip = q.clip > 0.f;
      const long long step_j = q.transposed ? q.ldo : 1;
      float* const row = q.transposed ? q.out + prow : q.out + prow * q.ldo;
      if (q.accumulate) {  // all old values loaded before any store: one round trip
        float prev[R];
#pragma unroll
        for (int j = 0; j < R; ++j) prev[j] = j < q.r ? row[j * step_j] : 0.f;
#pragma unroll
        for (int j = 0; j < R; ++j) {
          float v = acc[j];
          if (clip) v = fminf(fmaxf(v, -q.clip), q.clip);
          if (j < q.r) row[j * step_j] = prev[j] + v;
        }
      } else {
#pragma unroll
        for (int j = 0; j < R; ++j) {
          float v = acc[j];
          if (clip) v = fminf(fmaxf(v, -q.clip), q.clip);
          if (j < q.r) row[j * step_j] = v;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols(R));
  }
}

template <class K>
bool set_smem_attr(K kern, size_t bytes) {
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess) {
    set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    return false;
  }
  return true;
}

template <int R, bool kBF16>
int launch_rank_typed(const RankArgs& a, cudaStream_t stream) {
  CUtensorMap tx, tl;
  if (!make_tmap_2d_16b(&tx, a.x, a.K, a.M, a.ldx, kBK, 128)) return MLORA_ERR_INVALID_ARG;
  if (!make_tmap_2d_16b(&tl, a.l, a.K, a.r, a.ldl, kBK, R)) return MLORA_ERR_INVALID_ARG;
  RankParams p;
  p.M = a.M;
  p.r = static_cast<int>(a.r);
  p.num_kb = static_cast<int>((a.K + kBK - 1) / kBK);
  p.splits = a.splits;
  p.scale = a.scale;
  p.out_rows = a.out_rows;
  p.ld_rows = a.ld_rows;
  p.out_t = a.out_t;
  p.ld_t = a.ld_t;
  p.split_out = a.split_out ? 1 : 0;
  p.split_pattern = a.split_pattern;
  p.partials = a.partials;
  p.counters = a.counters;
  p.status = device_status_ptr();
  p.row_group = a.row_group;
  p.group_cols = a.group_cols > 0 ? static_cast<int>(a.group_cols) : R;
  auto kern = rank_proj_kernel<R, kBF16>;
  if (!set_smem_attr(kern, smem_bytes(R))) return MLORA_ERR_CUDA;
  dim3 grid(static_cast<unsigned>((a.M + 127) / 128), static_cast<unsigned>(a.splits));
  LaunchScope scope(kKindRank, stream);
  kern<<<grid, kThreads, smem_bytes(R), stream>>>(tx, tl, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("rank launch: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

template <int R, bool kBF16>
int launch_wgrad_typed(const WgradArgs* probs, int n, cudaStream_t stream) {
  CUtensorMap tb[2], ts[2];
  WgradParams p;
  p.nprobs = n;
  int total = 0;
  for (int i = 0; i < 2; ++i) {
    const WgradArgs& a = probs[i < n ? i : 0];
    if (!make_tmap_2d_16b(&tb[i], a.big, a.P, a.M, a.ldb, 64, kBK)) return MLORA_ERR_INVALID_ARG;
    if (!make_tmap_2d_16b(&ts[i], a.st, a.M, a.R, a.ld_st, kBK, R)) return MLORA_ERR_INVALID_ARG;
    WgradProblem& q = p.prob[i];
    q.M = a.M;
    q.P = a.P;
    q.r = static_cast<int>(a.r);
    q.num_kb = static_cast<int>((a.M + kBK - 1) / kBK);
    q.splits = a.splits;
    q.tiles = static_cast<int>((a.P + 127) / 128);
    q.out = a.out;
    q.ldo = a.ldo;
    q.transposed = a.transposed ? 1 : 0;
    q.accumulate = a.accumulate ? 1 : 0;
    q.clip = a.clip;
    q.partials = a.partials;
    q.counters = a.counters;
    if (i < n) total += q.tiles * q.splits;
    if (i == 0) p.ctas0 = q.tiles * q.splits;
  }
  p.status = device_status_ptr();
  auto kern = wgrad_kernel<R, kBF16>;
  if (!set_smem_attr(kern, smem_bytes(R))) return MLORA_ERR_CUDA;
  LaunchScope scope(kKindWgrad, stream);
  kern<<<total, kThreads, smem_bytes(R), stream>>>(tb[0], ts[0], tb[1], ts[1], p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("wgrad launch: ") + cudaGetErrorString(e));
    return MLORA_ERR_CUDA;
  }
  return MLORA_OK;
}

#define MLORA_DISPATCH_R(R_, FN, ...)                              \
  switch (R_) {                                                    \
    case 16: return FN<16, kB>(__VA_ARGS__);                       \
    case 32: return FN<32, kB>(__VA_ARGS__);                       \
    case 64: return FN<64, kB>(__VA_ARGS__);                       \
    case 128: return FN<128, kB>(__VA_ARGS__);                     \
    case 256: return FN<256, kB>(__VA_ARGS__);                     \
    default: set_error("unsupported padded rank"); return MLORA_ERR_UNSUPPORTED; \
  }

template <bool kB>
int rank_dispatch(const RankArgs& a, cudaStream_t s) {
  MLORA_DISPATCH_R(a.R, launch_rank_typed, a, s)
}

template <bool kB>
int wgrad_dispatch(const WgradArgs* probs, int n, cudaStream_t s) {
  MLORA_DISPATCH_R(probs[0].R, launch_wgrad_typed, probs, n, s)
}

}  // namespace

// Split counts keep tiles x splits within one wave of resident CTAs (2 per SM):
// a second, nearly empty wave would double the kernel's time.
int rank_splits(int64_t M, int64_t K) {
  const int64_t tiles = (M + 127) / 128;
  const int64_t num_kb = (K + kBK - 1) / kBK;
  int64_t splits = (2 * num_sms()) / tiles;
  const int64_t max_splits = num_kb / 4 > 0 ? num_kb / 4 : 1;  // >= 4 k-blocks per split
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  return static_cast<int>(splits);
}

int wgrad_splits(int64_t M, int64_t P, int nproblems) {
  const int64_t tiles = (P + 127) / 128 * nproblems;
  const int64_t num_kb = (M + kBK - 1) / kBK;
  int64_t splits = (2 * num_sms()) / tiles;
  const int64_t max_splits = num_kb / 4 > 0 ? num_kb / 4 : 1;
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  return static_cast<int>(splits);
}

int launch_rank(const RankArgs& a, cudaStream_t stream) {
  return a.elt == Elt::kBF16 ? rank_dispatch<true>(a, stream) : rank_dispatch<false>(a, stream);
}

int launch_wgrad(const WgradArgs* probs, int nprobs, cudaStream_t stream) {
  if (nprobs < 1 || nprobs > 2) return MLORA_ERR_INVALID_ARG;
  return probs[0].elt == Elt::kBF16 ? wgrad_dispatch<true>(probs, nprobs, stream)
                                    : wgrad_dispatch<false>(probs, nprobs, stream);
}

}  // namespace mlora
