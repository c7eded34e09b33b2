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
// along the reduction dimension across the CTAs of one thread-block cluster;
// their fp32 partial tiles are summed through distributed shared memory in
// fixed split order (cluster_reduce below), so results are bitwise
// reproducible and no global scratch or counter is needed.
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
constexpr int kMaxSplits = 8;                      // portable cluster size

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

// Cross-CTA split reduction through distributed shared memory.  The S CTAs of
// a cluster computed the same [128 x R] tile over S disjoint ranges of the
// reduction dimension (cluster rank = range index).  Each CTA parks its fp32
// partial in its own shared memory (the TMA stage area, free once the MMAs
// are done), column-major [j][row] so warps touch consecutive words; after a
// cluster barrier CTA c sums its slice of columns [c W, (c+1) W) (W = CP / S)
// of all 128 rows over s = 0..S-1 in that order -- fixed order, so results are
// bitwise reproducible -- and hands pairs of columns to `emit(j, v_j, v_j+1)`.
// A second barrier keeps every CTA resident until its peers have read it.
// Columns go in passes of CP (R > 128: two passes), each read from TMEM at
// `taddr` (this thread's lane) when `have` (zeros otherwise).  Every thread of
// the CTA calls this; only epilogue threads (`epi`) move data.
__host__ __device__ constexpr int reduce_cols(int R) { return R <= 128 ? R : 128; }

template <int R, typename Emit>
__device__ __forceinline__ void cluster_reduce(uint32_t taddr, bool have, float* buf, int S,
                                               uint32_t crank, int row_local, bool epi,
                                               Emit&& emit) {
  constexpr int CP = reduce_cols(R);
#pragma unroll 1
  for (int pass = 0; pass < R / CP; ++pass) {
    if (epi) {
      float acc[CP];
      if (have) {
        load_acc_row<CP>(taddr + pass * CP, acc);
      } else {
#pragma unroll
        for (int j = 0; j < CP; ++j) acc[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < CP; ++j) buf[j * 128 + row_local] = acc[j];
    }
    cluster_sync();
    if (epi) {
      const int W = CP / S;
      const int j0 = static_cast<int>(crank) * W;
      const uint32_t base = smem_u32(buf) + static_cast<uint32_t>(row_local) * 4u;
      uint32_t peer[8];
#pragma unroll
      for (int s = 0; s < 8; ++s) peer[s] = s < S ? mapa_shared(base, static_cast<uint32_t>(s)) : 0u;
#pragma unroll 1
      for (int jj = 0; jj < W; jj += 2) {
        const uint32_t off0 = static_cast<uint32_t>(j0 + jj) * 512u;
        float a[8], b[8];
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          a[s] = s < S ? ld_shared_cluster_f32(peer[s] + off0) : 0.f;
          b[s] = s < S ? ld_shared_cluster_f32(peer[s] + off0 + 512u) : 0.f;
        }
        float v0 = 0.f, v1 = 0.f;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          v0 += a[s];
          v1 += b[s];
        }
        emit(pass * CP + j0 + jj, v0, v1);
      }
    }
    cluster_sync();
  }
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
  uint32_t* status;
  const int32_t* row_group;  // optional: keep only columns [g*group_cols, (g+1)*group_cols)
  int group_cols;
};

// Grid (tiles, splits), cluster (1, splits, 1): the splits of one 128-row tile
// are one cluster.
template <int R, bool kBF16>
__global__ void __launch_bounds__(kThreads, 2)
    rank_proj_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_l,
                     const RankParams p) {
  using T = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
  constexpr int S = num_stages(R);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S * stage_bytes(R));
  uint64_t* empty_bar = full_bar + S;
  uint64_t* done_bar = empty_bar + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

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
  // A programmatic dependent launch gets here while the previous kernel may
  // still run: nothing is read before it has completed (a no-op otherwise).
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const int tile = blockIdx.x;
  const uint32_t crank = cluster_ctarank();
  const SplitWork w = split_work(tile, static_cast<int>(crank), p.splits, p.num_kb);
  const bool has_work = w.kb_begin < w.kb_end;
  if (has_work) {
    run_pipeline<R, false, kBF16>(smem, full_bar, empty_bar, done_bar, tmem, &tm_x, &tm_l,
                                  tile * 128, w.kb_begin, w.kb_end, p.status);
  }
  // a programmatic dependent (the weight-gradient kernel) may start its set-up
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const bool epi = warp >= 2;
  const int row_local = static_cast<int>((warp & 3u) * 32 + lane_id());
  const long long row = static_cast<long long>(tile) * 128 + row_local;
  bool have = false;
  if (epi && has_work) {
    have = mbar_wait(done_bar, 0, p.status, kDevTimeoutAccFull);
    tc_fence_after();
  }
  int group = -1;
  if (epi && p.row_group != nullptr && row < p.M) group = p.row_group[row];
  const bool live = epi && row < p.M;
  auto emit = [&](int j, float v0, float v1) {
    if (!live) return;
    v0 *= p.scale;
    v1 *= p.scale;
    if (p.split_out) {
      // fp32 path: bf16 hi/lo parts of the scaled value (bf16 instantiation only)
      const float h0 = __bfloat162float(__float2bfloat16_rn(v0));
      const float h1 = __bfloat162float(__float2bfloat16_rn(v1));
      for (int s = 0; s < 3; ++s) {
        const bool lo = (p.split_pattern >> s) & 1u;
        const float o0 = lo ? v0 - h0 : v0, o1 = lo ? v1 - h1 : v1;
        if (p.out_rows != nullptr)
          *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(p.out_rows) +
                                       row * p.ld_rows + s * R + j) = pack2<__nv_bfloat16>(o0, o1);
        if (p.out_t != nullptr) {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out_t) + s * p.M + row;
          dst[static_cast<long long>(j) * p.ld_t] = __float2bfloat16_rn(o0);
          dst[static_cast<long long>(j + 1) * p.ld_t] = __float2bfloat16_rn(o1);
        }
      }
      return;
    }
    if (p.row_group != nullptr) {
      // stacked adapters: the row keeps only its own adapter's columns (an
      // id outside [0, R / group_cols) keeps none)
      if (j / p.group_cols != group) v0 = 0.f;
      if ((j + 1) / p.group_cols != group) v1 = 0.f;
    }
    if (p.out_rows != nullptr)
      *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(p.out_rows) + row * p.ld_rows + j) =
          pack2<T>(v0, v1);
    if (p.out_t != nullptr) {
      T* dst = reinterpret_cast<T*>(p.out_t) + row;
      dst[static_cast<long long>(j) * p.ld_t] = static_cast<T>(v0);
      dst[static_cast<long long>(j + 1) * p.ld_t] = static_cast<T>(v1);
    }
  };
  cluster_reduce<R>(tmem + ((static_cast<uint32_t>(row_local & ~31)) << 16), have,
                    reinterpret_cast<float*>(smem), p.splits, crank, row_local, epi, emit);
  // zero padding of the row buffer past the computed columns (cluster rank 0)
  if (live && crank == 0 && p.out_rows != nullptr) {
    const long long from = p.split_out ? 3 * R : R;
    if (p.split_out) {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out_rows) + row * p.ld_rows;
      for (long long j = from; j < p.ld_rows; j += 8)
        *reinterpret_cast<uint4*>(dst + j) = make_uint4(0, 0, 0, 0);
    } else {
      T* dst = reinterpret_cast<T*>(p.out_rows) + row * p.ld_rows;
      for (long long j = from; j < p.ld_rows; j += 8)
        *reinterpret_cast<uint4*>(dst + j) = make_uint4(0, 0, 0, 0);
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
  int r, num_kb, tiles;
  float* out;     // fp32, or 16-bit (the operands' type) when out16
  long long ldo;
  int transposed;
  int accumulate;
  int out16;
  float clip;
};

struct WgradParams {
  WgradProblem prob[2];
  int nprobs;
  int splits;  // cluster size: the splits of one tile are one cluster
  int ctas0;   // CTAs of problem 0 (= tiles * splits)
  uint32_t* status;
};

// 1-D grid, cluster (splits, 1, 1): CTA b of problem q works on tile
// b / splits over token range b % splits (= its cluster rank).
template <int R, bool kBF16>
__global__ void __launch_bounds__(kThreads, 2)
    wgrad_kernel(const __grid_constant__ CUtensorMap tm_big0, const __grid_constant__ CUtensorMap tm_st0,
                 const __grid_constant__ CUtensorMap tm_big1, const __grid_constant__ CUtensorMap tm_st1,
                 const WgradParams p) {
  constexpr int S = num_stages(R);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S * stage_bytes(R));
  uint64_t* empty_bar = full_bar + S;
  uint64_t* done_bar = empty_bar + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

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
  // nothing is read before a programmatic predecessor has completed
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const int which = (static_cast<int>(blockIdx.x) < p.ctas0) ? 0 : 1;
  const WgradProblem& q = p.prob[which];
  const int local = static_cast<int>(blockIdx.x) - (which ? p.ctas0 : 0);
  const uint32_t crank = cluster_ctarank();
  const int tile = local / p.splits;
  const SplitWork w = split_work(tile, static_cast<int>(crank), p.splits, q.num_kb);
  const bool has_work = w.kb_begin < w.kb_end;
  if (has_work) {
    run_pipeline<R, true, kBF16>(smem, full_bar, empty_bar, done_bar, tmem,
                                 which ? &tm_big1 : &tm_big0, which ? &tm_st1 : &tm_st0,
                                 tile * 128, w.kb_begin, w.kb_end, p.status);
  }
  // a programmatic dependent (the dx GEMM, which reads none of this kernel's
  // outputs) may start on the SMs this grid frees during its reduction tail
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const bool epi = warp >= 2;
  const int row_local = static_cast<int>((warp & 3u) * 32 + lane_id());
  const long long prow = static_cast<long long>(tile) * 128 + row_local;
  bool have = false;
  if (epi && has_work) {
    have = mbar_wait(done_bar, 0, p.status, kDevTimeoutAccFull);
    tc_fence_after();
  }
  const bool live = epi && prow < q.P;
  const bool clip = q.clip > 0.f;
  const long long step_j = q.transposed ? q.ldo : 1;
  const long long row_off = q.transposed ? prow : prow * q.ldo;
  float* const out_row = q.out + row_off;
  using T = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
  auto emit = [&](int j, float v0, float v1) {
    if (!live) return;
    if (clip) {
      v0 = fminf(fmaxf(v0, -q.clip), q.clip);
      v1 = fminf(fmaxf(v1, -q.clip), q.clip);
    }
    const bool w0 = j < q.r, w1 = j + 1 < q.r;
    if (q.out16) {  // gradients in the operands' 16-bit type (sum kept in fp32)
      T* h0 = reinterpret_cast<T*>(q.out) + row_off + j * step_j;
      T* h1 = h0 + step_j;
      if (q.accumulate) {
        const float o0 = w0 ? static_cast<float>(*h0) : 0.f;
        const float o1 = w1 ? static_cast<float>(*h1) : 0.f;
        v0 += o0;
        v1 += o1;
      }
      if (w0) *h0 = static_cast<T>(v0);
      if (w1) *h1 = static_cast<T>(v1);
      return;
    }
    float* d0 = out_row + j * step_j;
    float* d1 = d0 + step_j;
    if (q.accumulate) {  // both old values loaded before either store
      const float o0 = w0 ? *d0 : 0.f, o1 = w1 ? *d1 : 0.f;
      if (w0) *d0 = o0 + v0;
      if (w1) *d1 = o1 + v1;
    } else {
      if (w0) *d0 = v0;
      if (w1) *d1 = v1;
    }
  };
  cluster_reduce<R>(tmem + ((static_cast<uint32_t>(row_local & ~31)) << 16), have,
                    reinterpret_cast<float*>(smem), p.splits, crank, row_local, epi, emit);
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

// Launches `kern` with a (cx, cy, 1) cluster; `overlap_prev` also makes it a
// programmatic dependent of the previous kernel on the stream.
template <typename Kern, typename... Args>
cudaError_t launch_clustered(Kern kern, dim3 grid, size_t smem, cudaStream_t stream, unsigned cx,
                             unsigned cy, bool overlap_prev, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cx;
  attr[0].val.clusterDim.y = cy;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = overlap_prev ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <int R, bool kBF16>
int launch_rank_typed(const RankArgs& a, cudaStream_t stream) {
  CUtensorMap tx, tl;
  if (!make_tmap_2d_16b(&tx, a.x, a.K, a.M, a.ldx, kBK, 128)) return MLORA_ERR_INVALID_ARG;
  if (!make_tmap_2d_16b(&tl, a.l, a.K, a.r, a.ldl, kBK, R)) return MLORA_ERR_INVALID_ARG;
  if (a.splits < 1 || a.splits > kMaxSplits || (a.splits & (a.splits - 1)) != 0) {
    set_error("rank: splits must be 1, 2, 4 or 8");
    return MLORA_ERR_INVALID_ARG;
  }
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
  p.status = device_status_ptr();
  p.row_group = a.row_group;
  p.group_cols = a.group_cols > 0 ? static_cast<int>(a.group_cols) : R;
  auto kern = rank_proj_kernel<R, kBF16>;
  if (!set_smem_attr(kern, smem_bytes(R))) return MLORA_ERR_CUDA;
  dim3 grid(static_cast<unsigned>((a.M + 127) / 128), static_cast<unsigned>(a.splits));
  LaunchScope scope(kKindRank, stream);
  cudaError_t e = launch_clustered(kern, grid, smem_bytes(R), stream, 1u,
                                   static_cast<unsigned>(a.splits), a.overlap_prev, tx, tl, p);
  if (e == cudaSuccess) e = cudaGetLastError();
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
  p.splits = probs[0].splits;
  if (p.splits < 1 || p.splits > kMaxSplits || (p.splits & (p.splits - 1)) != 0 ||
      (n == 2 && probs[1].splits != p.splits)) {
    set_error("wgrad: splits must be 1, 2, 4 or 8 and equal for both problems");
    return MLORA_ERR_INVALID_ARG;
  }
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
    q.tiles = static_cast<int>((a.P + 127) / 128);
    q.out = a.out;
    q.ldo = a.ldo;
    q.transposed = a.transposed ? 1 : 0;
    q.accumulate = a.accumulate ? 1 : 0;
    q.out16 = a.out16 ? 1 : 0;
    q.clip = a.clip;
    if (i < n) total += q.tiles * p.splits;
    if (i == 0) p.ctas0 = q.tiles * p.splits;
  }
  p.status = device_status_ptr();
  auto kern = wgrad_kernel<R, kBF16>;
  if (!set_smem_attr(kern, smem_bytes(R))) return MLORA_ERR_CUDA;
  LaunchScope scope(kKindWgrad, stream);
  cudaError_t e = launch_clustered(kern, dim3(static_cast<unsigned>(total)), smem_bytes(R), stream,
                                   static_cast<unsigned>(p.splits), 1u, probs[0].overlap_prev,
                                   tb[0], ts[0], tb[1], ts[1], p);
  if (e == cudaSuccess) e = cudaGetLastError();
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

int pow2_splits(int64_t tiles, int64_t num_kb) {
  int64_t cap = (2 * num_sms()) / tiles;
  const int64_t max_splits = num_kb / 4 > 0 ? num_kb / 4 : 1;  // >= 4 k-blocks per split
  if (cap > max_splits) cap = max_splits;
  int splits = 1;
  while (splits * 2 <= cap && splits * 2 <= kMaxSplits) splits *= 2;
  return splits;
}

}  // namespace

// Split counts (the cluster size of the split reduction: 1, 2, 4 or 8) keep
// tiles x splits within one wave of resident CTAs (2 per SM): a second, nearly
// empty wave would double the kernel's time.
int rank_splits(int64_t M, int64_t K) {
  return pow2_splits((M + 127) / 128, (K + kBK - 1) / kBK);
}

int wgrad_splits(int64_t M, int64_t P, int nproblems) {
  return pow2_splits((P + 127) / 128 * nproblems, (M + kBK - 1) / kBK);
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
