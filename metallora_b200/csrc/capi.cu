// C-ABI layer: argument validation, workspace planning, tensor-map encoding and
// the launch sequences of the LoRA-linear operations.  See
// include/metallora_b200.h for the contract of each entry point.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <initializer_list>
#include <mutex>
#include <string>
#include <vector>

#include "internal.h"
#include "../../include/metallora_b200.h"

// Per-device status word written by kernels whose bounded waits ran out.
__device__ uint32_t g_mlora_device_status;

namespace mlora {

namespace {
thread_local std::string t_last_error;
constexpr int kMaxDevices = 64;

struct DeviceInfo {
  std::once_flag once;
  int sms = 0;
  int major = 0;
  uint32_t* status = nullptr;
  cudaError_t err = cudaSuccess;
};
DeviceInfo g_dev[kMaxDevices];

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

DeviceInfo& dev_info() {
  const int d = current_device();
  DeviceInfo& info = g_dev[d < kMaxDevices ? d : 0];
  std::call_once(info.once, [&info, d]() {
    cudaDeviceProp prop;
    info.err = cudaGetDeviceProperties(&prop, d);
    if (info.err != cudaSuccess) return;
    info.sms = prop.multiProcessorCount;
    info.major = prop.major;
    void* p = nullptr;
    info.err = cudaGetSymbolAddress(&p, g_mlora_device_status);
    if (info.err != cudaSuccess) return;
    info.status = static_cast<uint32_t*>(p);
  });
  return info;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int64_t pad16(int64_t r) { return (r + 15) / 16 * 16; }
// Padded rank R handled by the tensor-core kernels (a power of two >= 16).
int64_t rank_tile(int64_t r) {
  int64_t R = 16;
  while (R < r) R *= 2;
  return R;
}
int64_t pad64(int64_t v) { return (v + 63) / 64 * 64; }
int64_t pad8(int64_t v) { return (v + 7) / 8 * 8; }

// Bump allocator over a caller workspace (256-byte aligned regions).
struct Carve {
  uint8_t* base;
  size_t off = 0;
  explicit Carve(void* b) : base(static_cast<uint8_t*>(b)) {}
  void* take(size_t bytes) {
    off = align_up(off, 256);
    void* p = base ? base + off : nullptr;
    off += bytes;
    return p;
  }
};

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int check_device() {
  DeviceInfo& info = dev_info();
  if (info.err != cudaSuccess)
    return fail(MLORA_ERR_CUDA, std::string("device query: ") + cudaGetErrorString(info.err));
  if (info.major != 10) return fail(MLORA_ERR_DEVICE, "device is not sm_100 (B200 class)");
  return MLORA_OK;
}

// need_n8: N is the row length of an operand read by TMA (backward: dy).
int check_shapes(int64_t M, int64_t K, int64_t N, int64_t r, int dtype, bool need_n8 = true) {
  if (M <= 0 || K <= 0 || N <= 0) return fail(MLORA_ERR_INVALID_ARG, "M, K, N must be positive");
  if (r < 1 || r > 256) return fail(MLORA_ERR_INVALID_ARG, "rank must be in [1, 256]");
  if (dtype != MLORA_DTYPE_BF16 && dtype != MLORA_DTYPE_F16 && dtype != MLORA_DTYPE_F32)
    return fail(MLORA_ERR_UNSUPPORTED, "dtype must be BF16, F16 or F32");
  if (K % 8 || r % 8)
    return fail(MLORA_ERR_UNSUPPORTED, "K and r must be multiples of 8 (16-byte rows)");
  if (need_n8 && N % 8)
    return fail(MLORA_ERR_UNSUPPORTED, "N must be a multiple of 8 for the backward (16-byte rows of dy)");
  if (M > (int64_t(1) << 31) - 1 || K > (1 << 24) || N > (1 << 24))
    return fail(MLORA_ERR_UNSUPPORTED, "shape too large");
  return MLORA_OK;
}

// ---- forward plan --------------------------------------------------------
struct FwdPlan {
  int64_t R, R64;
  int splits;
  void* xa_rows;
  void* xa_t;
  size_t bytes;
};

FwdPlan plan_forward(void* ws, int64_t M, int64_t K, int64_t r, bool need_xa_t) {
  FwdPlan p;
  p.R = rank_tile(r);
  p.R64 = pad64(p.R);
  p.splits = rank_splits(M, K);
  Carve c(ws);
  p.xa_rows = c.take(static_cast<size_t>(M) * p.R64 * 2);
  p.xa_t = need_xa_t ? c.take(static_cast<size_t>(p.R) * pad8(M) * 2) : nullptr;
  p.bytes = align_up(c.off, 256);
  return p;
}

// ---- backward plan -------------------------------------------------------
struct BwdPlan {
  int64_t R, R64;
  int rsplits, wsplits;
  void* bt;
  void* u_rows;
  void* u_t;
  void* xa_t;
  size_t bytes;
};

BwdPlan plan_backward(void* ws, int64_t M, int64_t K, int64_t N, int64_t r, bool need_xa_t) {
  BwdPlan p;
  p.R = rank_tile(r);
  p.R64 = pad64(p.R);
  p.rsplits = rank_splits(M, N > K ? N : K);
  p.wsplits = wgrad_splits(M, N > K ? N : K, 2);
  Carve c(ws);
  p.bt = c.take(static_cast<size_t>(p.R) * N * 2);
  p.u_rows = c.take(static_cast<size_t>(M) * p.R64 * 2);
  p.u_t = c.take(static_cast<size_t>(p.R) * pad8(M) * 2);
  p.xa_t = need_xa_t ? c.take(static_cast<size_t>(p.R) * pad8(M) * 2) : nullptr;
  p.bytes = align_up(c.off, 256);
  return p;
}

// ---- fp32 (split-precision) plans -----------------------------------------
// Every fp32 operand is copied once as bf16 hi/lo segments; a product of two
// fp32 tensors becomes one bf16 GEMM over a 3x longer reduction whose segment
// pairs are (hi,hi), (hi,lo), (lo,hi).
struct F32FwdPlan {
  int64_t R, R3_64;
  int splits;
  void* xs;     // [M, 3K]  (hi, hi, lo)
  void* ws;     // [N, 3K]  (hi, lo, hi)
  void* as;     // [r, 3K]  (hi, lo, hi)
  void* bs;     // [N, 3R]  (hi, lo, hi)
  void* t_rows; // [M, pad64(3R)] (hi, hi, lo) of s.x.A^T
  size_t bytes;
};

F32FwdPlan plan_forward_f32(void* ws, int64_t M, int64_t K, int64_t N, int64_t r, bool lora) {
  F32FwdPlan p;
  p.R = rank_tile(r);
  p.R3_64 = pad64(3 * p.R);
  p.splits = rank_splits(M, 3 * K);
  Carve c(ws);
  p.xs = c.take(static_cast<size_t>(M) * 3 * K * 2);
  p.ws = c.take(static_cast<size_t>(N) * 3 * K * 2);
  p.as = lora ? c.take(static_cast<size_t>(r) * 3 * K * 2) : nullptr;
  p.bs = lora ? c.take(static_cast<size_t>(N) * 3 * p.R * 2) : nullptr;
  p.t_rows = lora ? c.take(static_cast<size_t>(M) * p.R3_64 * 2) : nullptr;
  p.bytes = align_up(c.off, 256);
  return p;
}

struct F32BwdPlan {
  int64_t R, R3_64, ld3;
  int rsplits, wsplits;
  void* dys_cols;  // [M, 3N] HHL
  void* xs_cols;   // [M, 3K] HHL
  void* dy_rows;   // [3M, N] HHL
  void* x_rows;    // [3M, K] HHL
  void* w0_rows;   // [3N, K] HLH (dx only)
  void* bts;       // [R, 3N] HLH
  void* as_cols;   // [r, 3K] HLH
  void* as_rows;   // [3R, K] HHL (dx only)
  void* u_rows;    // [M, pad64(3R)] HLH (dx only)
  void* u_t;       // [R, ld3] HLH
  void* t_t;       // [R, ld3] HLH
  size_t bytes;
};

F32BwdPlan plan_backward_f32(void* ws, int64_t M, int64_t K, int64_t N, int64_t r, bool dx) {
  F32BwdPlan p;
  p.R = rank_tile(r);
  p.R3_64 = pad64(3 * p.R);
  p.ld3 = pad8(3 * M);
  const int64_t big = 3 * (N > K ? N : K);
  p.rsplits = rank_splits(M, big);
  p.wsplits = wgrad_splits(3 * M, N > K ? N : K, 2);
  Carve c(ws);
  p.dys_cols = c.take(static_cast<size_t>(M) * 3 * N * 2);
  p.xs_cols = c.take(static_cast<size_t>(M) * 3 * K * 2);
  p.dy_rows = c.take(static_cast<size_t>(3 * M) * N * 2);
  p.x_rows = c.take(static_cast<size_t>(3 * M) * K * 2);
  p.w0_rows = dx ? c.take(static_cast<size_t>(3 * N) * K * 2) : nullptr;
  p.bts = c.take(static_cast<size_t>(p.R) * 3 * N * 2);
  p.as_cols = c.take(static_cast<size_t>(r) * 3 * K * 2);
  p.as_rows = dx ? c.take(static_cast<size_t>(3 * p.R) * K * 2) : nullptr;
  p.u_rows = dx ? c.take(static_cast<size_t>(M) * p.R3_64 * 2) : nullptr;
  p.u_t = c.take(static_cast<size_t>(p.R) * p.ld3 * 2);
  p.t_t = c.take(static_cast<size_t>(p.R) * p.ld3 * 2);
  p.bytes = align_up(c.off, 256);
  return p;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MLORA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int check_ptrs16(std::initializer_list<const void*> ptrs) {
  for (const void* q : ptrs)
    if (q && !aligned16(q)) return fail(MLORA_ERR_INVALID_ARG, "tensor pointers must be 16-byte aligned");
  return MLORA_OK;
}

// ---- decode plan (M <= 16, bf16, K % 32 == 0) ------------------------------
struct GemvPlan {
  bool split;
  int ctas;
  float* st;
  float* partials;
  int64_t partial_floats;
  size_t bytes;
};

bool use_gemv(int64_t M, int64_t K, int dtype) {
  return M <= kGemvMaxTokens && K % 32 == 0 && dtype == MLORA_DTYPE_BF16;
}

GemvPlan plan_gemv(void* ws, int64_t M, int64_t K, int64_t N, int64_t r, int scheme,
                   int64_t group) {
  GemvPlan p;
  const DecodeConfig cfg = decode_config(scheme, M, N, K, r, group);
  p.split = cfg.split_blocks;
  p.ctas = cfg.ctas;
  Carve c(ws);
  p.st = static_cast<float*>(
      c.take(static_cast<size_t>(rank_small_splits(K)) * M * (r > 0 ? r : 1) * 4));
  p.partial_floats = p.split ? static_cast<int64_t>(p.ctas) * M * 128 : 0;
  p.partials = p.split ? static_cast<float*>(c.take(static_cast<size_t>(p.partial_floats) * 4))
                       : nullptr;
  p.bytes = align_up(c.off, 256);
  return p;
}

// Decode-size forward: sT = s.x.A^T (if a) with the partial flags zeroed,
// then the stream-K GEMV with the rank term (a programmatic dependent).
int run_gemv(int scheme, const void* x, const void* w, const void* scales_t,
             int64_t group, const void* a, const void* b, void* y, int64_t M, int64_t K,
             int64_t N, int64_t r, float alpha, void* workspace, size_t workspace_bytes,
             cudaStream_t s, int64_t ldy = 0) {
  const GemvPlan need = plan_gemv(nullptr, M, K, N, r, scheme, group);
  if (workspace == nullptr || workspace_bytes < need.bytes)
    return fail(MLORA_ERR_WORKSPACE, "decode workspace needs " + std::to_string(need.bytes) + " bytes");
  const GemvPlan p = plan_gemv(workspace, M, K, N, r, scheme, group);
  // partial slots: set to their empty pattern by the rank kernel when there
  // is one, else by a small fill kernel; the decode kernel is the
  // programmatic dependent of either.  No shared row block uses none.
  int rc;
  if (a == nullptr && p.split && (rc = launch_partials_fill(p.partials, p.partial_floats, s)))
    return rc;
  if (a != nullptr &&
      (rc = launch_rank_small(x, a, M, K, r, alpha / static_cast<float>(r), p.st, p.partials,
                              p.partial_floats, s)))
    return rc;
  GemvArgs g;
  g.scheme = scheme;
  g.x = x;
  g.w = w;
  g.scales_t = scales_t;
  g.b = a != nullptr ? b : nullptr;
  g.st = p.st;
  g.y = y;
  g.partials = p.partials;
  g.M = M;
  g.N = N;
  g.K = K;
  g.r = r;
  g.group = group;
  g.ldy = ldy;
  g.pdl = a != nullptr || p.split;
  return launch_gemv(g, s);
}

int lora_forward_f32(const float* x, const float* w0, const float* a, const float* b, float* y,
                     int64_t M, int64_t K, int64_t N, int64_t r, float alpha, void* workspace,
                     size_t workspace_bytes, cudaStream_t s) {
  const bool lora = a != nullptr;
  const F32FwdPlan need = plan_forward_f32(nullptr, M, K, N, r, lora);
  if (workspace == nullptr || workspace_bytes < need.bytes || !aligned16(workspace))
    return fail(MLORA_ERR_WORKSPACE, "fp32 forward workspace needs " + std::to_string(need.bytes) + " bytes");
  const F32FwdPlan p = plan_forward_f32(workspace, M, K, N, r, lora);
  int rc;
  if ((rc = launch_split3_cols(x, M, K, K, p.xs, K, 3 * K, kHHL, s))) return rc;
  if ((rc = launch_split3_cols(w0, N, K, K, p.ws, K, 3 * K, kHLH, s))) return rc;
  GemmArgs ga;
  ga.x = p.xs;
  ga.w = p.ws;
  ga.d = y;
  ga.M = M;
  ga.N = N;
  ga.K = 3 * K;
  ga.ldx = 3 * K;
  ga.ldw = 3 * K;
  ga.ldd = N;
  ga.w_mn_major = false;
  ga.elt = Elt::kBF16;
  ga.out_dtype = MLORA_DTYPE_F32;
  if (lora) {
    if ((rc = launch_split3_cols(a, r, K, K, p.as, K, 3 * K, kHLH, s))) return rc;
    if ((rc = launch_split3_cols(b, N, r, r, p.bs, p.R, 3 * p.R, kHLH, s))) return rc;
    RankArgs ra;
    ra.x = p.xs;
    ra.l = p.as;
    ra.M = M;
    ra.K = 3 * K;
    ra.r = r;
    ra.R = p.R;
    ra.ldx = 3 * K;
    ra.ldl = 3 * K;
    ra.scale = alpha / static_cast<float>(r);
    ra.out_rows = p.t_rows;
    ra.ld_rows = p.R3_64;
    ra.out_t = nullptr;
    ra.ld_t = 0;
    ra.split_out = true;
    ra.split_pattern = kHHL;
    ra.splits = p.splits;
    ra.elt = Elt::kBF16;
    if ((rc = launch_rank(ra, s))) return rc;
    ga.x2 = p.t_rows;
    ga.w2 = p.bs;
    ga.R = 3 * p.R;
    ga.w2_rows = 3 * p.R;
    ga.ldx2 = p.R3_64;
    ga.ldw2 = 3 * p.R;
  }
  return launch_gemm(ga, s);
}

int lora_backward_f32(const float* dy, const float* x, const float* w0, const float* a,
                      const float* b, float* dx, float* da, float* db, int64_t M, int64_t K,
                      int64_t N, int64_t r, float alpha, float clip, bool accumulate,
                      void* workspace, size_t workspace_bytes, cudaStream_t s) {
  const bool want_dx = dx != nullptr;
  const F32BwdPlan need = plan_backward_f32(nullptr, M, K, N, r, want_dx);
  if (workspace == nullptr || workspace_bytes < need.bytes || !aligned16(workspace))
    return fail(MLORA_ERR_WORKSPACE, "fp32 backward workspace needs " + std::to_string(need.bytes) + " bytes");
  const F32BwdPlan p = plan_backward_f32(workspace, M, K, N, r, want_dx);
  const int64_t tm = (M + 127) / 128, tn = (N + 127) / 128;
  const float scale = alpha / static_cast<float>(r);
  int rc;
  if ((rc = launch_split3_cols(dy, M, N, N, p.dys_cols, N, 3 * N, kHHL, s))) return rc;
  if ((rc = launch_split3_cols(x, M, K, K, p.xs_cols, K, 3 * K, kHHL, s))) return rc;
  if ((rc = launch_split3_rows(dy, M, N, N, p.dy_rows, M, kHHL, s))) return rc;
  if ((rc = launch_split3_rows(x, M, K, K, p.x_rows, M, kHHL, s))) return rc;
  if ((rc = launch_split3_cols_t(b, N, r, r, p.bts, p.R, N, 3 * N, kHLH, s))) return rc;
  if ((rc = launch_split3_cols(a, r, K, K, p.as_cols, K, 3 * K, kHLH, s))) return rc;

  // s.dy.B (hi, lo, hi): rows feed the dx GEMM, the transpose feeds dA.
  RankArgs ru;
  ru.x = p.dys_cols;
  ru.l = p.bts;
  ru.M = M;
  ru.K = 3 * N;
  ru.r = p.R;
  ru.R = p.R;
  ru.ldx = 3 * N;
  ru.ldl = 3 * N;
  ru.scale = scale;
  ru.out_rows = want_dx ? p.u_rows : nullptr;
  ru.ld_rows = p.R3_64;
  ru.out_t = p.u_t;
  ru.ld_t = p.ld3;
  ru.split_out = true;
  ru.split_pattern = kHLH;
  ru.splits = rank_splits(M, 3 * N);
  if (ru.splits > p.rsplits) ru.splits = p.rsplits;
  ru.elt = Elt::kBF16;
  if ((rc = launch_rank(ru, s))) return rc;
  // s.x.A^T (hi, lo, hi) transposed: feeds dB.
  RankArgs rt = ru;
  rt.x = p.xs_cols;
  rt.l = p.as_cols;
  rt.K = 3 * K;
  rt.r = r;
  rt.ldx = 3 * K;
  rt.ldl = 3 * K;
  rt.out_rows = nullptr;
  rt.out_t = p.t_t;
  rt.splits = rank_splits(M, 3 * K);
  if (rt.splits > p.rsplits) rt.splits = p.rsplits;
  if ((rc = launch_rank(rt, s))) return rc;

  if (want_dx) {
    if ((rc = launch_split3_rows(w0, N, K, K, p.w0_rows, N, kHLH, s))) return rc;
    if ((rc = launch_split3_rows(a, r, K, K, p.as_rows, p.R, kHHL, s))) return rc;
    GemmArgs ga;
    ga.x = p.dys_cols;
    ga.w = p.w0_rows;
    ga.x2 = p.u_rows;
    ga.w2 = p.as_rows;
    ga.d = dx;
    ga.M = M;
    ga.N = K;
    ga.K = 3 * N;
    ga.R = 3 * p.R;
    ga.w2_rows = 3 * p.R;
    ga.ldx = 3 * N;
    ga.ldw = K;
    ga.ldx2 = p.R3_64;
    ga.ldw2 = K;
    ga.ldd = K;
    ga.w_mn_major = true;
    ga.elt = Elt::kBF16;
    ga.out_dtype = MLORA_DTYPE_F32;
    if ((rc = launch_gemm(ga, s))) return rc;
  }

  WgradArgs w[2];
  w[0].big = p.dy_rows;
  w[0].st = p.t_t;
  w[0].ld_st = p.ld3;
  w[0].M = 3 * M;
  w[0].P = N;
  w[0].r = r;
  w[0].R = p.R;
  w[0].ldb = N;
  w[0].out = db;
  w[0].ldo = r;
  w[0].transposed = false;
  w[0].accumulate = accumulate;
  w[0].clip = clip;
  w[0].splits = p.wsplits;
  w[0].elt = Elt::kBF16;
  w[1] = w[0];
  w[1].big = p.x_rows;
  w[1].st = p.u_t;
  w[1].P = K;
  w[1].ldb = K;
  w[1].out = da;
  w[1].ldo = K;
  w[1].transposed = true;
  return launch_wgrad(w, 2, s);
}

// Phases of the 16-bit backward (flags MLORA_BWD_DEFER_DX / MLORA_BWD_DX_ONLY).
constexpr int kPhaseAll = 0, kPhaseDeferDx = 1, kPhaseDx = 2;

// Backward of the 16-bit LoRA linear (dense W0, or a quantised W0 described
// by qdx): rank projections, dA/dB weight gradients, dx GEMM.
int backward16(const void* dy, const void* x, const void* w0, const QGemmArgs* qdx,
               const void* a, const void* b, const void* saved_xa, void* dx, float* da,
               float* db, int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
               float clip_value, bool accumulate, int dtype, void* workspace,
               size_t workspace_bytes, cudaStream_t s, int phase = kPhaseAll,
               bool grads16 = false) {
  int rc;
  const BwdPlan need = plan_backward(nullptr, M, K, N, r, saved_xa == nullptr);
  if (workspace == nullptr || workspace_bytes < need.bytes || !aligned16(workspace))
    return fail(MLORA_ERR_WORKSPACE, "backward workspace needs " + std::to_string(need.bytes) + " bytes");
  const BwdPlan p = plan_backward(workspace, M, K, N, r, saved_xa == nullptr);
  const Elt elt = dtype == MLORA_DTYPE_BF16 ? Elt::kBF16 : Elt::kF16;
  const float scale = alpha / static_cast<float>(r);

  // kPhaseDeferDx stops before the dx GEMM (s.dy.B stays in the workspace);
  // kPhaseDx runs only that GEMM, from the workspace of a deferred call.
  if (phase != kPhaseDx) {
    // B^T, zero-padded to R rows: the K-major operand of the U = s.dy.B projection.
    if ((rc = launch_transpose_pad(b, N, r, r, p.bt, p.R, elt, s))) return rc;

    RankArgs ra;
    ra.x = dy;
    ra.l = p.bt;
    ra.M = M;
    ra.K = N;
    ra.r = p.R;
    ra.R = p.R;
    ra.ldx = N;
    ra.ldl = N;
    ra.scale = scale;
    ra.out_rows = dx ? p.u_rows : nullptr;
    ra.ld_rows = p.R64;
    ra.out_t = p.u_t;
    ra.ld_t = pad8(M);
    ra.splits = rank_splits(M, N);
    ra.elt = elt;
    ra.overlap_prev = true;  // set-up overlaps the transpose just launched
    if (ra.splits > p.rsplits) ra.splits = p.rsplits;
    if ((rc = launch_rank(ra, s))) return rc;
    ra.overlap_prev = false;

    const void* xa_t = saved_xa;
    if (xa_t == nullptr) {
      RankArgs rt = ra;
      rt.x = x;
      rt.l = a;
      rt.K = K;
      rt.r = r;
      rt.ldx = K;
      rt.ldl = K;
      rt.out_rows = nullptr;
      rt.out_t = p.xa_t;
      rt.splits = rank_splits(M, K);
      if (rt.splits > p.rsplits) rt.splits = p.rsplits;
      if ((rc = launch_rank(rt, s))) return rc;
      xa_t = p.xa_t;
    }

    // Weight gradients first: they read dy right after the rank pass over it
    // (much of dy still in L2); the compute-bound dx GEMM follows.
    WgradArgs w[2];
    // db[n, j] = sum_m dy[m, n] * (s x A^T)[m, j]
    w[0].big = dy;
    w[0].st = xa_t;
    w[0].ld_st = pad8(M);
    w[0].M = M;
    w[0].P = N;
    w[0].r = r;
    w[0].R = p.R;
    w[0].ldb = N;
    w[0].out = db;
    w[0].ldo = r;
    w[0].transposed = false;
    w[0].accumulate = accumulate;
    w[0].out16 = grads16;
    w[0].overlap_prev = true;  // set-up overlaps the rank projection before it
    w[0].clip = clip_value;
    w[0].splits = p.wsplits;
    w[0].elt = elt;
    // da[j, k] = sum_m (s dy B)[m, j] * x[m, k]
    w[1] = w[0];
    w[1].big = x;
    w[1].st = p.u_t;
    w[1].P = K;
    w[1].ldb = K;
    w[1].out = da;
    w[1].ldo = K;
    w[1].transposed = true;
    if ((rc = launch_wgrad(w, 2, s))) return rc;
  }
  if (phase == kPhaseDeferDx) return MLORA_OK;

  if (dx != nullptr && qdx != nullptr) {
    QGemmArgs q = *qdx;
    q.w_mn_major = true;
    q.x = dy;
    q.x2 = p.u_rows;
    q.up = a;
    q.d = dx;
    q.M = M;
    q.N = K;
    q.K = N;
    q.R = p.R;
    q.ldx = N;
    q.ldx2 = p.R64;
    q.ldd = K;
    q.up_rows = r;
    q.up_ld = K;
    q.up_cols = K;
    if ((rc = launch_qgemm(q, s))) return rc;
  } else if (dx != nullptr) {
    GemmArgs ga;
    ga.x = dy;
    ga.w = w0;
    ga.x2 = p.u_rows;
    ga.w2 = a;
    ga.d = dx;
    ga.M = M;
    ga.N = K;  // output columns of dx
    ga.K = N;  // reduction over out_features
    ga.R = p.R;
    ga.w2_rows = r;
    ga.ldx = N;
    ga.ldw = K;
    ga.ldx2 = p.R64;
    ga.ldw2 = K;
    ga.ldd = K;
    ga.w_mn_major = true;
    ga.elt = elt;
    ga.out_dtype = dtype;
    // in one call the weight-gradient kernel was launched just before: the
    // GEMM starts on SMs it frees; its X2 (s.dy.B) was complete before that
    // kernel passed its own wait, and dy, W0 before the call
    ga.overlap_prev = phase == kPhaseAll;
    if ((rc = launch_gemm(ga, s))) return rc;
  }

  return MLORA_OK;
}

// ---- plain linear and merge plans ----------------------------------------
size_t linear_ws(int64_t M, int64_t K, int64_t N, int dtype) {
  if (use_gemv(M, K, dtype)) return plan_gemv(nullptr, M, K, N, 0, 0, 64).bytes;
  if (dtype != MLORA_DTYPE_F32) return 0;
  return plan_forward_f32(nullptr, M, K, N, 1, false).bytes;
}

size_t merge_ws(int64_t N, int64_t K, int64_t r, int dtype) {
  if (dtype != MLORA_DTYPE_F32) return 0;
  const int64_t r8 = pad8(r);
  return align_up(static_cast<size_t>(N) * 3 * r8 * 2, 256) +
         align_up(static_cast<size_t>(3 * r8) * K * 2, 256);
}

// ---- launch accounting / profiling ---------------------------------------
std::atomic<long long> g_launches{0};
std::mutex g_prof_mu;
bool g_prof_on = false;
struct ProfRec {
  int kind;
  cudaEvent_t start, stop;
};
std::vector<ProfRec> g_prof_recs;
std::vector<cudaEvent_t> g_event_pool;

cudaEvent_t pool_event() {
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

}  // namespace

LaunchScope::LaunchScope(int kind, cudaStream_t stream) : kind_(kind), stream_(stream) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  std::lock_guard<std::mutex> lock(g_prof_mu);
  if (!g_prof_on) return;
  cudaEvent_t start = pool_event();
  stop_ = pool_event();
  if (start == nullptr || stop_ == nullptr) return;
  cudaEventRecord(start, stream_);
  g_prof_recs.push_back({kind_, start, stop_});
}

LaunchScope::~LaunchScope() {
  if (stop_ != nullptr) cudaEventRecord(stop_, stream_);
}

void set_error(const std::string& msg) { t_last_error = msg; }

bool make_tmap_2d_16b(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  return make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, base, inner, outer,
                      row_stride_elems * 2, box_inner, box_outer, true);
}

bool make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, uint32_t esize, const void* base,
                  uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                  uint32_t box_outer, bool swizzle128) {
  (void)esize;
  auto fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled entry point unavailable");
    return false;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) +
              ") for dims " + std::to_string(inner) + "x" + std::to_string(outer) + " box " +
              std::to_string(box_inner) + "x" + std::to_string(box_outer));
    return false;
  }
  return true;
}

uint32_t* device_status_ptr() { return dev_info().status; }
int num_sms() {
  const int s = dev_info().sms;
  return s > 0 ? s : 148;
}

}  // namespace mlora

using namespace mlora;

extern "C" {

int mlora_version(void) { return 100; }

const char* mlora_status_string(int status) {
  switch (status) {
    case MLORA_OK: return "ok";
    case MLORA_ERR_INVALID_ARG: return "invalid argument";
    case MLORA_ERR_UNSUPPORTED: return "unsupported";
    case MLORA_ERR_CUDA: return "CUDA error";
    case MLORA_ERR_WORKSPACE: return "workspace too small";
    case MLORA_ERR_DEVICE: return "unsupported device";
    default: return "unknown status";
  }
}

const char* mlora_last_error_message(void) { return t_last_error.c_str(); }

int mlora_device_supported(int device) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return prop.major == 10 ? 1 : 0;
}

int mlora_device_status(uint32_t* out, int reset) {
  if (out == nullptr) return fail(MLORA_ERR_INVALID_ARG, "out is NULL");
  int rc = check_device();
  if (rc) return rc;
  uint32_t v = 0;
  cudaError_t e = cudaMemcpy(&v, device_status_ptr(), 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && reset) e = cudaMemset(device_status_ptr(), 0, 4);
  if (e != cudaSuccess) return fail(MLORA_ERR_CUDA, std::string("status read: ") + cudaGetErrorString(e));
  *out = v;
  return MLORA_OK;
}

size_t mlora_lora_forward_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r, int dtype) {
  if (M <= 0 || K <= 0 || N <= 0 || r <= 0) return 0;
  if (dtype == MLORA_DTYPE_F32) return plan_forward_f32(nullptr, M, K, N, r, true).bytes;
  size_t bytes = plan_forward(nullptr, M, K, r, true).bytes;
  if (use_gemv(M, K, dtype)) bytes = std::max(bytes, plan_gemv(nullptr, M, K, N, r, 0, 64).bytes);
  return bytes;
}

namespace {
// 16-bit LoRA forward (decode kernel for <= 16 tokens without saved_xa, else
// rank kernel + tcgen05 GEMM) writing y rows with stride ldy.
int lora_forward16(const void* x, const void* w0, const void* a, const void* b, void* y,
                   int64_t ldy, void* saved_xa, int64_t M, int64_t K, int64_t N, int64_t r,
                   float alpha, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  int rc;
  if (saved_xa == nullptr && use_gemv(M, K, dtype))
    return run_gemv(0, x, w0, nullptr, 64, a, b, y, M, K, N, r, alpha, workspace,
                    workspace_bytes, static_cast<cudaStream_t>(stream), ldy);
  const FwdPlan need = plan_forward(nullptr, M, K, r, saved_xa == nullptr);
  if (workspace == nullptr || workspace_bytes < need.bytes || !aligned16(workspace))
    return fail(MLORA_ERR_WORKSPACE, "forward workspace needs " + std::to_string(need.bytes) + " bytes");
  const FwdPlan p = plan_forward(workspace, M, K, r, saved_xa == nullptr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const Elt elt = dtype == MLORA_DTYPE_BF16 ? Elt::kBF16 : Elt::kF16;

  RankArgs ra;
  ra.x = x;
  ra.l = a;
  ra.M = M;
  ra.K = K;
  ra.r = r;
  ra.R = p.R;
  ra.ldx = K;
  ra.ldl = K;
  ra.scale = alpha / static_cast<float>(r);
  ra.out_rows = p.xa_rows;
  ra.ld_rows = p.R64;
  ra.out_t = saved_xa ? saved_xa : p.xa_t;
  ra.ld_t = pad8(M);
  ra.splits = p.splits;
  ra.elt = elt;
  if ((rc = launch_rank(ra, s))) return rc;

  GemmArgs ga;
  ga.x = x;
  ga.w = w0;
  ga.x2 = p.xa_rows;
  ga.w2 = b;
  ga.d = y;
  ga.M = M;
  ga.N = N;
  ga.K = K;
  ga.R = p.R;
  ga.w2_rows = r;
  ga.ldx = K;
  ga.ldw = K;
  ga.ldx2 = p.R64;
  ga.ldw2 = r;
  ga.ldd = ldy;
  ga.w_mn_major = false;
  ga.elt = elt;
  ga.out_dtype = dtype;
  ga.overlap_prev = true;  // only X2 (s.x.A^T) comes from the rank kernel just launched
  return launch_gemm(ga, s);
}
}  // namespace

int mlora_lora_forward(const void* x, const void* w0, const void* a, const void* b, void* y,
                       void* saved_xa, int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                       int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_shapes(M, K, N, r, dtype, false);
  if (rc) return rc;
  if (!x || !w0 || !a || !b || !y) return fail(MLORA_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(x) || !aligned16(w0) || !aligned16(a) || !aligned16(b) || !aligned16(y) ||
      (saved_xa && !aligned16(saved_xa)))
    return fail(MLORA_ERR_INVALID_ARG, "tensor pointers must be 16-byte aligned");
  if ((rc = check_device())) return rc;
  if (dtype == MLORA_DTYPE_F32) {
    if (saved_xa) return fail(MLORA_ERR_UNSUPPORTED, "saved_xa is not produced for F32");
    return lora_forward_f32(static_cast<const float*>(x), static_cast<const float*>(w0),
                            static_cast<const float*>(a), static_cast<const float*>(b),
                            static_cast<float*>(y), M, K, N, r, alpha, workspace, workspace_bytes,
                            static_cast<cudaStream_t>(stream));
  }
  return lora_forward16(x, w0, a, b, y, N, saved_xa, M, K, N, r, alpha, dtype, workspace,
                        workspace_bytes, stream);
}

size_t mlora_lora_backward_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r, int dtype) {
  if (M <= 0 || K <= 0 || N <= 0 || r <= 0) return 0;
  if (dtype == MLORA_DTYPE_F32) return plan_backward_f32(nullptr, M, K, N, r, true).bytes;
  return plan_backward(nullptr, M, K, N, r, true).bytes;
}

int mlora_lora_backward(const void* dy, const void* x, const void* w0, const void* a,
                        const void* b, const void* saved_xa, void* dx, float* da, float* db,
                        int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                        float clip_value, int dtype, void* workspace, size_t workspace_bytes,
                        void* stream) {
  return mlora_lora_backward_ex(dy, x, w0, a, b, saved_xa, dx, da, db, M, K, N, r, alpha,
                                clip_value, dtype, 0, workspace, workspace_bytes, stream);
}

int mlora_lora_backward_ex(const void* dy, const void* x, const void* w0, const void* a,
                           const void* b, const void* saved_xa, void* dx, float* da, float* db,
                           int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                           float clip_value, int dtype, int flags, void* workspace,
                           size_t workspace_bytes, void* stream) {
  const bool accumulate = (flags & MLORA_BWD_ACCUMULATE) != 0;
  if (flags & ~(MLORA_BWD_ACCUMULATE | MLORA_BWD_DEFER_DX | MLORA_BWD_DX_ONLY |
                MLORA_BWD_GRADS_16BIT))
    return fail(MLORA_ERR_INVALID_ARG, "unknown flags");
  const bool grads16 = (flags & MLORA_BWD_GRADS_16BIT) != 0;
  if (grads16 && dtype == MLORA_DTYPE_F32)
    return fail(MLORA_ERR_INVALID_ARG, "MLORA_BWD_GRADS_16BIT needs a 16-bit dtype");
  if ((flags & MLORA_BWD_DEFER_DX) && (flags & MLORA_BWD_DX_ONLY))
    return fail(MLORA_ERR_INVALID_ARG, "MLORA_BWD_DEFER_DX and MLORA_BWD_DX_ONLY exclude each other");
  const int phase = (flags & MLORA_BWD_DEFER_DX) ? kPhaseDeferDx
                    : (flags & MLORA_BWD_DX_ONLY) ? kPhaseDx : kPhaseAll;
  int rc = check_shapes(M, K, N, r, dtype);
  if (rc) return rc;
  if (!dy || !x || !a || !b || !da || !db) return fail(MLORA_ERR_INVALID_ARG, "NULL tensor pointer");
  if ((dx == nullptr) != (w0 == nullptr))
    return fail(MLORA_ERR_INVALID_ARG, "w0 and dx must be both set or both NULL");
  if (phase != kPhaseAll && (dx == nullptr || dtype == MLORA_DTYPE_F32))
    return fail(MLORA_ERR_INVALID_ARG, "a split backward needs dx and a 16-bit dtype");
  const void* ptrs[] = {dy, x, w0, a, b, saved_xa, dx, da, db};
  for (const void* q : ptrs)
    if (q && !aligned16(q)) return fail(MLORA_ERR_INVALID_ARG, "tensor pointers must be 16-byte aligned");
  if ((rc = check_device())) return rc;
  if (dtype == MLORA_DTYPE_F32)
    return lora_backward_f32(static_cast<const float*>(dy), static_cast<const float*>(x),
                             static_cast<const float*>(w0), static_cast<const float*>(a),
                             static_cast<const float*>(b), static_cast<float*>(dx), da, db, M, K,
                             N, r, alpha, clip_value, accumulate, workspace, workspace_bytes,
                             static_cast<cudaStream_t>(stream));
  return backward16(dy, x, w0, nullptr, a, b, saved_xa, dx, da, db, M, K, N, r, alpha, clip_value,
                    accumulate, dtype, workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                    phase, grads16);
}

long long mlora_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int mlora_profile_enable(int on) {
  std::lock_guard<std::mutex> lock(g_prof_mu);
  g_prof_on = on != 0;
  return MLORA_OK;
}

int mlora_profile_read(double* total_ms, long long* launches, int nkinds, int reset) {
  if (total_ms == nullptr || launches == nullptr || nkinds <= 0)
    return fail(MLORA_ERR_INVALID_ARG, "NULL output");
  std::lock_guard<std::mutex> lock(g_prof_mu);
  for (int k = 0; k < nkinds; ++k) total_ms[k] = 0.0, launches[k] = 0;
  for (const ProfRec& r : g_prof_recs) {
    float ms = 0.f;
    cudaError_t e = cudaEventSynchronize(r.stop);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, r.start, r.stop);
    if (e != cudaSuccess) return cuda_fail(e, "profile event");
    if (r.kind < nkinds) total_ms[r.kind] += ms, launches[r.kind] += 1;
  }
  if (reset) {
    for (const ProfRec& r : g_prof_recs) {
      g_event_pool.push_back(r.start);
      g_event_pool.push_back(r.stop);
    }
    g_prof_recs.clear();
  }
  return MLORA_OK;
}

// ---- optimizer ---------------------------------------------------------------

int mlora_adamw_step(void* param, float* grad, float* m, float* v, const float* state, int64_t n,
                     float lr, float beta1, float beta2, float eps, float weight_decay,
                     int param_dtype, const float* grad_scale, void* stream) {
  if (!param || !grad || !m || !v || !state) return fail(MLORA_ERR_INVALID_ARG, "NULL pointer");
  if (n <= 0) return fail(MLORA_ERR_INVALID_ARG, "n must be positive");
  if (param_dtype < MLORA_DTYPE_BF16 || param_dtype > MLORA_DTYPE_F32)
    return fail(MLORA_ERR_UNSUPPORTED, "param dtype must be BF16, F16 or F32");
  int rc = check_device();
  if (rc) return rc;
  return launch_adamw(param, param_dtype, grad, m, v, state, n, lr, beta1, beta2, eps,
                      weight_decay, grad_scale, 0, static_cast<cudaStream_t>(stream));
}

int mlora_sgd_step(void* param, float* grad, int64_t n, float lr, int param_dtype,
                   const float* grad_scale, void* stream) {
  if (!param || !grad) return fail(MLORA_ERR_INVALID_ARG, "NULL pointer");
  if (n <= 0) return fail(MLORA_ERR_INVALID_ARG, "n must be positive");
  if (param_dtype < MLORA_DTYPE_BF16 || param_dtype > MLORA_DTYPE_F32)
    return fail(MLORA_ERR_UNSUPPORTED, "param dtype must be BF16, F16 or F32");
  int rc = check_device();
  if (rc) return rc;
  // m, v and state are not touched in SGD mode.
  return launch_adamw(param, param_dtype, grad, nullptr, nullptr, nullptr, n, lr, 0.f, 0.f, 0.f,
                      0.f, grad_scale, 1, static_cast<cudaStream_t>(stream));
}

int mlora_adam_state_step(float* state, float beta1, float beta2, void* stream) {
  if (!state) return fail(MLORA_ERR_INVALID_ARG, "NULL state");
  int rc = check_device();
  if (rc) return rc;
  return launch_adam_state_step(state, beta1, beta2, static_cast<cudaStream_t>(stream));
}

size_t mlora_grad_norm_workspace_bytes(void) {
  return 256 + align_up(static_cast<size_t>(2 * 1024) * 4, 256);
}

int mlora_grad_norm_clip(const float* grad, int64_t n, float max_norm, float* out,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (!grad || !out) return fail(MLORA_ERR_INVALID_ARG, "NULL pointer");
  if (n <= 0) return fail(MLORA_ERR_INVALID_ARG, "n must be positive");
  int rc = check_device();
  if (rc) return rc;
  if (norm_grid() > 2 * 1024) return fail(MLORA_ERR_UNSUPPORTED, "too many SMs");
  if (!workspace || workspace_bytes < mlora_grad_norm_workspace_bytes() || !aligned16(workspace))
    return fail(MLORA_ERR_WORKSPACE, "grad-norm workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t* counter = static_cast<uint32_t*>(workspace);
  float* partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256);
  cudaError_t e = cudaMemsetAsync(counter, 0, 4, s);
  if (e != cudaSuccess) return cuda_fail(e, "memset");
  return launch_grad_norm(grad, n, max_norm, partials, counter, out, s);
}

// ---- quantised base weights ----------------------------------------------------

namespace {
int check_quant(int scheme, int64_t N, int64_t K, int64_t group) {
  if (scheme != MLORA_QUANT_NF4 && scheme != MLORA_QUANT_INT4 && scheme != MLORA_QUANT_INT8)
    return fail(MLORA_ERR_INVALID_ARG, "scheme must be NF4, INT4 or INT8");
  if (N <= 0 || K <= 0 || group <= 0) return fail(MLORA_ERR_INVALID_ARG, "N, K, group must be positive");
  if (scheme != MLORA_QUANT_INT8 && (K % 2))
    return fail(MLORA_ERR_INVALID_ARG, "4-bit codes pack two per byte: K must be even");
  return MLORA_OK;
}
}  // namespace

int mlora_quantize(const void* w, int w_dtype, int64_t N, int64_t K, int scheme, int64_t group,
                   void* codes, void* scales, void* zeros, void* stream) {
  int rc = check_quant(scheme, N, K, group);
  if (rc) return rc;
  if (!w || !codes || !scales || (scheme != MLORA_QUANT_NF4 && !zeros))
    return fail(MLORA_ERR_INVALID_ARG, "NULL pointer");
  if (w_dtype < MLORA_DTYPE_BF16 || w_dtype > MLORA_DTYPE_F32)
    return fail(MLORA_ERR_INVALID_ARG, "weight dtype must be BF16, F16 or F32");
  if ((rc = check_device())) return rc;
  return launch_quantize(w, w_dtype, N, K, scheme, group, codes, scales, zeros,
                         static_cast<cudaStream_t>(stream));
}

int mlora_dequantize(int scheme, const void* codes, const void* scales, const void* zeros,
                     int64_t N, int64_t K, int64_t group, void* out, int out_dtype, void* stream) {
  int rc = check_quant(scheme, N, K, group);
  if (rc) return rc;
  if (!codes || !scales || !out || (scheme != MLORA_QUANT_NF4 && !zeros))
    return fail(MLORA_ERR_INVALID_ARG, "NULL pointer");
  if (out_dtype < MLORA_DTYPE_BF16 || out_dtype > MLORA_DTYPE_F32)
    return fail(MLORA_ERR_INVALID_ARG, "out dtype must be BF16, F16 or F32");
  if ((rc = check_device())) return rc;
  return launch_dequantize(scheme, codes, scales, zeros, N, K, group, out, out_dtype,
                           static_cast<cudaStream_t>(stream));
}

namespace {
int check_qlora(int scheme, int64_t M, int64_t K, int64_t N, int64_t r, int64_t group, int dtype) {
  int rc = check_shapes(M, K, N, r, dtype);
  if (rc) return rc;
  if ((rc = check_quant(scheme, N, K, group))) return rc;
  if (dtype != MLORA_DTYPE_BF16)
    return fail(MLORA_ERR_UNSUPPORTED, "quantised-base paths take BF16 activations");
  if (group != 64 && group != 128 && group != 256)
    return fail(MLORA_ERR_UNSUPPORTED, "tensor-core quantised paths take group 64, 128 or 256");
  if (scheme != MLORA_QUANT_INT8 ? (K % 32) : (K % 16))
    return fail(MLORA_ERR_UNSUPPORTED, "code rows must be a multiple of 16 bytes (K % 32 for 4-bit)");
  return MLORA_OK;
}

size_t qscales_bytes(int64_t N, int64_t K, int64_t group) {
  return align_up(static_cast<size_t>((K + group - 1) / group) * prepared_ld(N) * 4, 256);
}

// The prepared scale table: per-row scales re-laid as [groups, prepared_ld(N)]
// (fp32 absmax, or (scale, zero) fp16 pairs), so a TMA box of it is a block of
// rows' scales for a range of k.
int prep_scales(int scheme, const void* scales, const void* zeros, int64_t N, int64_t K,
                int64_t group, void* scales_t, cudaStream_t s) {
  const int64_t G = (K + group - 1) / group;
  if (scheme == MLORA_QUANT_NF4)
    return launch_transpose_f32(static_cast<const float*>(scales), N, G, prepared_ld(N),
                                static_cast<float*>(scales_t), s);
  return launch_pack_scale_zero(scales, zeros, N, G, prepared_ld(N), scales_t, s);
}
}  // namespace

// Two ways to run a quantised base on the tensor cores:
//  * staged (default): one HBM-bound pass dequantises W into a bf16 [N, K]
//    copy at the front of the workspace (2.5 B/weight for 4-bit; ~18 us for
//    11008 x 4096), then the dense kernels run on it.  The fused kernel
//    dequantises each weight once per 128-token tile instead, so staging wins
//    from the first tile on.
//  * lean: the fused kernel dequantises inside its main loop and no dense copy
//    is made; chosen when the caller's workspace is below the staged size but
//    at least mlora_qlora_lean_workspace_bytes().
// Both give bitwise-identical results (the operands are bf16(dequant(W)) either way).
namespace {
size_t staged_w_bytes(int64_t N, int64_t K) { return align_up(static_cast<size_t>(N * K) * 2, 256); }

size_t qfwd_lean_bytes(int64_t M, int64_t K, int64_t N, int64_t r, int scheme, int64_t group) {
  size_t bytes = plan_forward(nullptr, M, K, r, true).bytes + qscales_bytes(N, K, group);
  if (use_gemv(M, K, MLORA_DTYPE_BF16))
    bytes = std::max(bytes, plan_gemv(nullptr, M, K, N, r, scheme, group).bytes + qscales_bytes(N, K, group));
  return bytes;
}

size_t qbwd_lean_bytes(int64_t M, int64_t K, int64_t N, int64_t r, int64_t group) {
  return plan_backward(nullptr, M, K, N, r, true).bytes + qscales_bytes(N, K, group);
}
}  // namespace

size_t mlora_qlora_lean_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r, int scheme,
                                        int64_t group, int backward) {
  if (M <= 0 || K <= 0 || N <= 0 || r <= 0 || group <= 0) return 0;
  return backward ? qbwd_lean_bytes(M, K, N, r, group) : qfwd_lean_bytes(M, K, N, r, scheme, group);
}

size_t mlora_qlora_forward_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r, int scheme,
                                           int64_t group) {
  (void)scheme;
  if (M <= 0 || K <= 0 || N <= 0 || r <= 0 || group <= 0) return 0;
  const size_t staged = staged_w_bytes(N, K) + plan_forward(nullptr, M, K, r, true).bytes;
  return std::max(staged, qfwd_lean_bytes(M, K, N, r, scheme, group));
}

size_t mlora_qlora_prepared_scales_bytes(int scheme, int64_t N, int64_t K, int64_t group) {
  if (N <= 0 || K <= 0 || group <= 0) return 0;
  (void)scheme;
  return qscales_bytes(N, K, group);
}

int mlora_qlora_prepare_scales(int scheme, const void* scales, const void* zeros, int64_t N,
                               int64_t K, int64_t group, void* out, void* stream) {
  int rc = check_quant(scheme, N, K, group);
  if (rc) return rc;
  if (!scales || !out || (scheme != MLORA_QUANT_NF4 && !zeros))
    return fail(MLORA_ERR_INVALID_ARG, "NULL pointer");
  if ((rc = check_ptrs16({scales, zeros, out}))) return rc;
  if ((rc = check_device())) return rc;
  return prep_scales(scheme, scales, zeros, N, K, group, out, static_cast<cudaStream_t>(stream));
}

int mlora_qlora_forward(const void* x, int scheme, const void* codes, const void* scales,
                        const void* zeros, int64_t group, const void* a, const void* b, void* y,
                        void* saved_xa, int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                        int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  return mlora_qlora_forward_ex(x, scheme, codes, scales, zeros, nullptr, group, a, b, y, saved_xa,
                                M, K, N, r, alpha, dtype, workspace, workspace_bytes, stream);
}

int mlora_qlora_forward_ex(const void* x, int scheme, const void* codes, const void* scales,
                           const void* zeros, const void* prepared, int64_t group, const void* a,
                           const void* b, void* y, void* saved_xa, int64_t M, int64_t K, int64_t N,
                           int64_t r, float alpha, int dtype, void* workspace,
                           size_t workspace_bytes, void* stream) {
  int rc = check_qlora(scheme, M, K, N, r, group, dtype);
  if (rc) return rc;
  if (!x || !codes || !scales || !a || !b || !y || (scheme != MLORA_QUANT_NF4 && !zeros))
    return fail(MLORA_ERR_INVALID_ARG, "NULL tensor pointer");
  if ((rc = check_ptrs16({x, codes, scales, zeros, prepared, a, b, y, saved_xa, workspace})))
    return rc;
  if ((rc = check_device())) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (saved_xa == nullptr && use_gemv(M, K, dtype)) {
    const void* table = prepared;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    size_t ws_bytes = workspace_bytes;
    if (table == nullptr) {  // build the scale table in the workspace
      const size_t sb = qscales_bytes(N, K, group);
      if (ws == nullptr || ws_bytes < sb)
        return fail(MLORA_ERR_WORKSPACE, "decode workspace too small for the scale table");
      if ((rc = prep_scales(scheme, scales, zeros, N, K, group, ws, s))) return rc;
      table = ws;
      ws += sb;
      ws_bytes -= sb;
    }
    return run_gemv(scheme, x, codes, table, group, a, b, y, M, K, N, r, alpha, ws, ws_bytes, s);
  }
  const size_t wbytes = staged_w_bytes(N, K);
  const size_t staged = wbytes + plan_forward(nullptr, M, K, r, saved_xa == nullptr).bytes;
  if (workspace != nullptr && workspace_bytes >= staged) {
    if ((rc = launch_dequantize(scheme, codes, scales, zeros, N, K, group, workspace,
                                MLORA_DTYPE_BF16, s)))
      return rc;
    return mlora_lora_forward(x, workspace, a, b, y, saved_xa, M, K, N, r, alpha, dtype,
                              static_cast<uint8_t*>(workspace) + wbytes, workspace_bytes - wbytes,
                              stream);
  }
  const size_t sbytes = qscales_bytes(N, K, group);
  const FwdPlan need = plan_forward(nullptr, M, K, r, saved_xa == nullptr);
  if (workspace == nullptr || workspace_bytes < need.bytes + sbytes)
    return fail(MLORA_ERR_WORKSPACE, "qlora forward workspace needs " + std::to_string(staged) +
                                         " bytes (or " + std::to_string(need.bytes + sbytes) +
                                         " for the lean fused-dequant kernel)");
  const FwdPlan p = plan_forward(workspace, M, K, r, saved_xa == nullptr);
  const void* scales_t = prepared;
  if (scales_t == nullptr) {
    void* tab = static_cast<uint8_t*>(workspace) + p.bytes;
    if ((rc = prep_scales(scheme, scales, zeros, N, K, group, tab, s))) return rc;
    scales_t = tab;
  }
  RankArgs ra;
  ra.x = x;
  ra.l = a;
  ra.M = M;
  ra.K = K;
  ra.r = r;
  ra.R = p.R;
  ra.ldx = K;
  ra.ldl = K;
  ra.scale = alpha / static_cast<float>(r);
  ra.out_rows = p.xa_rows;
  ra.ld_rows = p.R64;
  ra.out_t = saved_xa ? saved_xa : p.xa_t;
  ra.ld_t = pad8(M);
  ra.splits = p.splits;
  ra.elt = Elt::kBF16;
  if ((rc = launch_rank(ra, s))) return rc;
  QGemmArgs q;
  q.scheme = scheme;
  q.w_mn_major = false;
  q.x = x;
  q.x2 = p.xa_rows;
  q.codes = codes;
  q.scales_t = scales_t;
  q.up = b;
  q.d = y;
  q.M = M;
  q.N = N;
  q.K = K;
  q.R = p.R;
  q.ldx = K;
  q.ldx2 = p.R64;
  q.ldd = N;
  q.group = group;
  q.up_rows = r;
  q.up_ld = r;
  q.up_cols = r;
  return launch_qgemm(q, s);
}

size_t mlora_qlora_backward_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r,
                                            int scheme, int64_t group) {
  (void)scheme;
  if (M <= 0 || K <= 0 || N <= 0 || r <= 0 || group <= 0) return 0;
  const size_t staged = staged_w_bytes(N, K) + plan_backward(nullptr, M, K, N, r, true).bytes;
  return std::max(staged, qbwd_lean_bytes(M, K, N, r, group));
}

int mlora_qlora_backward(const void* dy, const void* x, int scheme, const void* codes,
                         const void* scales, const void* zeros, int64_t group, const void* a,
                         const void* b, const void* saved_xa, void* dx, float* da, float* db,
                         int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                         float clip_value, int dtype, int flags, void* workspace,
                         size_t workspace_bytes, void* stream) {
  return mlora_qlora_backward_ex(dy, x, scheme, codes, scales, zeros, nullptr, group, a, b,
                                 saved_xa, dx, da, db, M, K, N, r, alpha, clip_value, dtype, flags,
                                 workspace, workspace_bytes, stream);
}

int mlora_qlora_backward_ex(const void* dy, const void* x, int scheme, const void* codes,
                            const void* scales, const void* zeros, const void* prepared,
                            int64_t group, const void* a, const void* b, const void* saved_xa,
                            void* dx, float* da, float* db, int64_t M, int64_t K, int64_t N,
                            int64_t r, float alpha, float clip_value, int dtype, int flags,
                            void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_qlora(scheme, M, K, N, r, group, dtype);
  if (rc) return rc;
  if (flags & ~MLORA_BWD_ACCUMULATE) return fail(MLORA_ERR_INVALID_ARG, "unknown flags");
  if (!dy || !x || !a || !b || !da || !db) return fail(MLORA_ERR_INVALID_ARG, "NULL tensor pointer");
  if (dx && (!codes || !scales || (scheme != MLORA_QUANT_NF4 && !zeros)))
    return fail(MLORA_ERR_INVALID_ARG, "dx needs the quantised weight");
  if ((rc = check_ptrs16({dy, x, codes, scales, zeros, prepared, a, b, saved_xa, dx, da, db,
                          workspace})))
    return rc;
  if ((rc = check_device())) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool accumulate = (flags & MLORA_BWD_ACCUMULATE) != 0;
  const size_t bytes = plan_backward(nullptr, M, K, N, r, saved_xa == nullptr).bytes;
  if (dx == nullptr)  // weight gradients only: the base weight is not read
    return backward16(dy, x, nullptr, nullptr, a, b, saved_xa, nullptr, da, db, M, K, N, r, alpha,
                      clip_value, accumulate, dtype, workspace, workspace_bytes, s);
  const size_t wbytes = staged_w_bytes(N, K);
  if (workspace != nullptr && workspace_bytes >= wbytes + bytes) {
    if ((rc = launch_dequantize(scheme, codes, scales, zeros, N, K, group, workspace,
                                MLORA_DTYPE_BF16, s)))
      return rc;
    return backward16(dy, x, workspace, nullptr, a, b, saved_xa, dx, da, db, M, K, N, r, alpha,
                      clip_value, accumulate, dtype, static_cast<uint8_t*>(workspace) + wbytes,
                      workspace_bytes - wbytes, s);
  }
  const size_t sbytes = qscales_bytes(N, K, group);
  if (workspace == nullptr || workspace_bytes < bytes + sbytes)
    return fail(MLORA_ERR_WORKSPACE, "qlora backward workspace needs " +
                                         std::to_string(wbytes + bytes) + " bytes (or " +
                                         std::to_string(bytes + sbytes) +
                                         " for the lean fused-dequant kernel)");
  const void* scales_t = prepared;
  if (scales_t == nullptr) {
    void* tab = static_cast<uint8_t*>(workspace) + bytes;
    if ((rc = prep_scales(scheme, scales, zeros, N, K, group, tab, s))) return rc;
    scales_t = tab;
  }
  QGemmArgs q;
  q.scheme = scheme;
  q.codes = codes;
  q.scales_t = scales_t;
  q.group = group;
  return backward16(dy, x, nullptr, &q, a, b, saved_xa, dx, da, db, M, K, N, r, alpha, clip_value,
                    accumulate, dtype, workspace, bytes, s);
}

size_t mlora_multi_lora_forward_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r,
                                                int64_t n, int dtype) {
  (void)N;
  (void)dtype;
  if (M <= 0 || K <= 0 || r <= 0 || n <= 0) return 0;
  return plan_forward(nullptr, M, K, n * r, false).bytes;
}

int mlora_multi_lora_forward(const void* x, const void* w0, const void* a_stack,
                             const void* b_stack, const int32_t* ids, void* y, int64_t M,
                             int64_t K, int64_t N, int64_t r, int64_t n, float alpha, int dtype,
                             void* workspace, size_t workspace_bytes, void* stream) {
  if (n < 1 || n * r > 256)
    return fail(MLORA_ERR_UNSUPPORTED, "stacked adapters: need 1 <= n and n * r <= 256");
  int rc = check_shapes(M, K, N, n * r, dtype, false);
  if (rc) return rc;
  if (dtype == MLORA_DTYPE_F32)
    return fail(MLORA_ERR_UNSUPPORTED, "multi-adapter forward takes BF16 or F16");
  if (!x || !a_stack || !b_stack || !ids || !y) return fail(MLORA_ERR_INVALID_ARG, "NULL tensor pointer");
  if ((rc = check_ptrs16({x, w0, a_stack, b_stack, y, workspace}))) return rc;
  if ((rc = check_device())) return rc;
  const int64_t R = n * r;
  const FwdPlan need = plan_forward(nullptr, M, K, R, false);
  if (workspace == nullptr || workspace_bytes < need.bytes)
    return fail(MLORA_ERR_WORKSPACE, "multi-adapter workspace needs " + std::to_string(need.bytes) + " bytes");
  const FwdPlan p = plan_forward(workspace, M, K, R, false);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const Elt elt = dtype == MLORA_DTYPE_BF16 ? Elt::kBF16 : Elt::kF16;
  // one pass over x projects onto every stacked adapter; each row keeps its own
  RankArgs ra;
  ra.x = x;
  ra.l = a_stack;
  ra.M = M;
  ra.K = K;
  ra.r = R;
  ra.R = p.R;
  ra.ldx = K;
  ra.ldl = K;
  ra.scale = alpha / static_cast<float>(r);
  ra.out_rows = p.xa_rows;
  ra.ld_rows = p.R64;
  ra.out_t = nullptr;
  ra.ld_t = 0;
  ra.splits = p.splits;
  ra.elt = elt;
  ra.row_group = ids;
  ra.group_cols = r;
  if ((rc = launch_rank(ra, s))) return rc;
  GemmArgs ga;
  ga.d = y;
  ga.M = M;
  ga.N = N;
  ga.ldd = N;
  ga.w_mn_major = false;
  ga.elt = elt;
  ga.out_dtype = dtype;
  if (w0 != nullptr) {  // y = [x | xa] . [w0 | b_stack]^T
    ga.x = x;
    ga.w = w0;
    ga.K = K;
    ga.ldx = K;
    ga.ldw = K;
    ga.x2 = p.xa_rows;
    ga.w2 = b_stack;
    ga.R = p.R;
    ga.w2_rows = R;
    ga.ldx2 = p.R64;
    ga.ldw2 = R;
  } else {  // LoRA term only: y = xa . b_stack^T
    ga.x = p.xa_rows;
    ga.w = b_stack;
    ga.K = R;
    ga.ldx = p.R64;
    ga.ldw = R;
  }
  return launch_gemm(ga, s);
}

namespace {
struct EmbedBwdPlan {
  FwdPlan rank;       // U = s dy.A^T rows [T, R64] (16-bit)
  void* gt;           // s B[idx]^T [R, pad8(T)]
  int wsplits;
  size_t bytes;
};

EmbedBwdPlan plan_embed_bwd(void* ws, int64_t T, int64_t D, int64_t r) {
  EmbedBwdPlan p;
  p.rank = plan_forward(ws, T, D, r, false);
  Carve c(ws == nullptr ? nullptr : static_cast<uint8_t*>(ws) + p.rank.bytes);
  p.gt = c.take(static_cast<size_t>(p.rank.R) * pad8(T) * 2);
  p.wsplits = wgrad_splits(T, D, 1);
  p.bytes = p.rank.bytes + align_up(c.off, 256);
  return p;
}

int check_embed(int64_t T, int64_t V, int64_t D, int64_t r, int dtype) {
  if (T <= 0 || V <= 0 || D <= 0) return fail(MLORA_ERR_INVALID_ARG, "T, V, D must be positive");
  if (r < 1 || r > 256) return fail(MLORA_ERR_INVALID_ARG, "rank must be in [1, 256]");
  if (dtype != MLORA_DTYPE_BF16 && dtype != MLORA_DTYPE_F16 && dtype != MLORA_DTYPE_F32)
    return fail(MLORA_ERR_UNSUPPORTED, "dtype must be BF16, F16 or F32");
  if (dtype != MLORA_DTYPE_F32 && (D % 8 || r % 8))
    return fail(MLORA_ERR_UNSUPPORTED, "16-bit embedding: D and r must be multiples of 8");
  if (T > (int64_t(1) << 31) - 1 || V > (int64_t(1) << 31) - 1)
    return fail(MLORA_ERR_UNSUPPORTED, "too many tokens or rows");
  return MLORA_OK;
}
}  // namespace

size_t mlora_lora_embedding_workspace_bytes(int64_t T, int64_t D, int64_t r, int dtype,
                                            int backward) {
  if (T <= 0 || D <= 0 || r <= 0) return 0;
  if (dtype == MLORA_DTYPE_F32) return backward ? align_up(static_cast<size_t>(T) * r * 4, 256) : 0;
  if (!backward) return align_up(static_cast<size_t>(T) * r * 2, 256);
  return plan_embed_bwd(nullptr, T, D, r).bytes;
}

int mlora_lora_embedding_forward(const int32_t* idx, const void* table, const void* a,
                                 const void* b, void* out, int64_t T, int64_t V, int64_t D,
                                 int64_t r, float alpha, int dtype, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  int rc = check_embed(T, V, D, r, dtype);
  if (rc) return rc;
  if (!idx || !table || !a || !b || !out) return fail(MLORA_ERR_INVALID_ARG, "NULL tensor pointer");
  if ((rc = check_ptrs16({table, a, b, out, workspace}))) return rc;
  if ((rc = check_device())) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float scale = alpha / static_cast<float>(r);
  if (dtype == MLORA_DTYPE_F32)
    return launch_embedding_f32(idx, static_cast<const float*>(table), static_cast<const float*>(a),
                                static_cast<const float*>(b), static_cast<float*>(out), T, V, D, r,
                                scale, s);
  const size_t need = align_up(static_cast<size_t>(T) * r * 2, 256);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(MLORA_ERR_WORKSPACE, "embedding workspace needs " + std::to_string(need) + " bytes");
  const Elt elt = dtype == MLORA_DTYPE_BF16 ? Elt::kBF16 : Elt::kF16;
  // G = B[idx] [T, r], then out = s * G.A + E[idx] on the tensor cores
  if ((rc = launch_gather_rows(idx, b, V, T, r, r, workspace, r, nullptr, 0, 1.f, elt, s))) return rc;
  GemmArgs ga;
  ga.x = workspace;
  ga.w = a;            // A [r, D] read MN-major as W [K = r, N = D]
  ga.d = out;
  ga.c = table;        // addend rows gathered by idx
  ga.ldc = D;
  ga.c_index = idx;
  ga.c_rows = V;
  ga.acc_scale = scale;
  ga.M = T;
  ga.N = D;
  ga.K = r;
  ga.ldx = r;
  ga.ldw = D;
  ga.ldd = D;
  ga.w_mn_major = true;
  ga.elt = elt;
  ga.out_dtype = dtype;
  return launch_gemm(ga, s);
}

int mlora_lora_embedding_backward(const void* dy, const int32_t* idx, const int32_t* sorted_idx,
                                  const int32_t* order, const void* a, const void* b, float* da,
                                  float* db, int64_t T, int64_t V, int64_t D, int64_t r,
                                  float alpha, int dtype, int flags, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  int rc = check_embed(T, V, D, r, dtype);
  if (rc) return rc;
  if (flags & ~MLORA_BWD_ACCUMULATE) return fail(MLORA_ERR_INVALID_ARG, "unknown flags");
  if (!dy || !idx || !sorted_idx || !order || !a || !b || !da || !db)
    return fail(MLORA_ERR_INVALID_ARG, "NULL tensor pointer");
  if ((rc = check_ptrs16({dy, a, b, da, db, workspace}))) return rc;
  if ((rc = check_device())) return rc;
  const bool accumulate = (flags & MLORA_BWD_ACCUMULATE) != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float scale = alpha / static_cast<float>(r);
  cudaError_t e;
  if (!accumulate) {  // rows of db no token touches are zero
    e = cudaMemsetAsync(db, 0, static_cast<size_t>(V) * r * 4, s);
    if (e != cudaSuccess) return cuda_fail(e, "memset");
  }
  if (dtype == MLORA_DTYPE_F32) {
    const size_t need = align_up(static_cast<size_t>(T) * r * 4, 256);
    if (workspace == nullptr || workspace_bytes < need)
      return fail(MLORA_ERR_WORKSPACE, "embedding backward workspace needs " + std::to_string(need) + " bytes");
    float* u = static_cast<float*>(workspace);
    if ((rc = launch_rows_dot_f32(static_cast<const float*>(dy), static_cast<const float*>(a), u, T,
                                  D, r, scale, s)))
      return rc;
    if ((rc = launch_segment_rows(sorted_idx, order, u, r, T, r, db, V, true, dtype, s))) return rc;
    return launch_embed_da_f32(idx, static_cast<const float*>(b), static_cast<const float*>(dy), da,
                               V, T, D, r, scale, accumulate, s);
  }
  const EmbedBwdPlan need = plan_embed_bwd(nullptr, T, D, r);
  if (workspace == nullptr || workspace_bytes < need.bytes)
    return fail(MLORA_ERR_WORKSPACE, "embedding backward workspace needs " + std::to_string(need.bytes) + " bytes");
  const EmbedBwdPlan p = plan_embed_bwd(workspace, T, D, r);
  const Elt elt = dtype == MLORA_DTYPE_BF16 ? Elt::kBF16 : Elt::kF16;
  // U = s dy.A^T, then dB rows as in-order sums of U over each index's tokens
  RankArgs ra;
  ra.x = dy;
  ra.l = a;
  ra.M = T;
  ra.K = D;
  ra.r = r;
  ra.R = p.rank.R;
  ra.ldx = D;
  ra.ldl = D;
  ra.scale = scale;
  ra.out_rows = p.rank.xa_rows;
  ra.ld_rows = p.rank.R64;
  ra.out_t = nullptr;
  ra.ld_t = 0;
  ra.splits = p.rank.splits;
  ra.elt = elt;
  if ((rc = launch_rank(ra, s))) return rc;
  if ((rc = launch_segment_rows(sorted_idx, order, p.rank.xa_rows, p.rank.R64, T, r, db, V, true,
                                dtype, s)))
    return rc;
  // dA = (s B[idx])^T . dy on the tensor cores (weight-gradient kernel)
  if ((rc = launch_gather_rows(idx, b, V, T, r, p.rank.R, nullptr, 0, p.gt, pad8(T), scale, elt, s)))
    return rc;
  WgradArgs w;
  w.big = dy;
  w.st = p.gt;
  w.ld_st = pad8(T);
  w.M = T;
  w.P = D;
  w.r = r;
  w.R = p.rank.R;
  w.ldb = D;
  w.out = da;
  w.ldo = D;
  w.transposed = true;
  w.accumulate = accumulate;
  w.clip = 0.f;
  w.splits = p.wsplits;
  w.elt = elt;
  return launch_wgrad(&w, 1, s);
}

size_t mlora_lora_kv_cache_workspace_bytes(int64_t batch, int64_t D_in, int64_t D_kv, int64_t r,
                                           int dtype) {
  return mlora_lora_forward_workspace_bytes(batch, D_in, D_kv, r, dtype);
}

int mlora_lora_kv_cache_update(const void* x, const void* wk, const void* wv, const void* ak,
                               const void* bk, const void* av, const void* bv, void* k_cache,
                               void* v_cache, int64_t batch, int64_t cur_pos, int64_t max_seq,
                               int64_t D_in, int64_t D_kv, int64_t r, float alpha, int dtype,
                               void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != MLORA_DTYPE_BF16 && dtype != MLORA_DTYPE_F16)
    return fail(MLORA_ERR_UNSUPPORTED, "KV-cache update takes BF16 or F16");
  int rc = check_shapes(batch, D_in, D_kv, r, dtype, false);
  if (rc) return rc;
  if (D_kv % 8) return fail(MLORA_ERR_UNSUPPORTED, "KV width must be a multiple of 8");
  if (max_seq <= 0 || cur_pos < 0 || cur_pos >= max_seq)
    return fail(MLORA_ERR_INVALID_ARG, "cur_pos must be in [0, max_seq)");
  if (!x || !wk || !wv || !ak || !bk || !av || !bv || !k_cache || !v_cache)
    return fail(MLORA_ERR_INVALID_ARG, "NULL tensor pointer");
  if ((rc = check_ptrs16({x, wk, wv, ak, bk, av, bv, k_cache, v_cache, workspace}))) return rc;
  if ((rc = check_device())) return rc;
  // row b of the new K (V) is cache[b, cur_pos, :]: row stride max_seq * D_kv
  const int64_t ld = max_seq * D_kv;
  const size_t off = static_cast<size_t>(cur_pos) * D_kv * 2;
  if ((rc = lora_forward16(x, wk, ak, bk, static_cast<uint8_t*>(k_cache) + off, ld, nullptr, batch,
                           D_in, D_kv, r, alpha, dtype, workspace, workspace_bytes, stream)))
    return rc;
  return lora_forward16(x, wv, av, bv, static_cast<uint8_t*>(v_cache) + off, ld, nullptr, batch,
                        D_in, D_kv, r, alpha, dtype, workspace, workspace_bytes, stream);
}

int mlora_peer_allreduce(const void* bufs, const void* flags, int rank, int world,
                         uint32_t seq, float* out, int64_t n, float scale, uint32_t* counter,
                         void* stream) {
  if (!bufs || !flags || !out || !counter) return fail(MLORA_ERR_INVALID_ARG, "NULL pointer");
  if (world < 1 || world > 64 || rank < 0 || rank >= world)
    return fail(MLORA_ERR_INVALID_ARG, "rank must be in [0, world), world in [1, 64]");
  if (seq == 0) return fail(MLORA_ERR_INVALID_ARG, "seq starts at 1");
  if (n <= 0) return fail(MLORA_ERR_INVALID_ARG, "n must be positive");
  int rc;
  if ((rc = check_ptrs16({out}))) return rc;
  if ((rc = check_device())) return rc;
  return launch_peer_allreduce(bufs, flags, rank, world, seq, out, n, scale, counter,
                               static_cast<cudaStream_t>(stream));
}

size_t mlora_linear_workspace_bytes(int64_t M, int64_t K, int64_t N, int dtype) {
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  return linear_ws(M, K, N, dtype);
}

int mlora_linear(const void* x, const void* w, void* y, int64_t M, int64_t K, int64_t N, int dtype,
                 void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_shapes(M, K, N, 8, dtype, false);
  if (rc) return rc;
  if (!x || !w || !y) return fail(MLORA_ERR_INVALID_ARG, "NULL tensor pointer");
  if ((rc = check_ptrs16({x, w, y, workspace}))) return rc;
  if ((rc = check_device())) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (use_gemv(M, K, dtype))
    return run_gemv(0, x, w, nullptr, 64, nullptr, nullptr, y, M, K, N, 0, 1.f, workspace,
                    workspace_bytes, s);
  if (dtype == MLORA_DTYPE_F32)
    return lora_forward_f32(static_cast<const float*>(x), static_cast<const float*>(w), nullptr,
                            nullptr, static_cast<float*>(y), M, K, N, 1, 1.f, workspace,
                            workspace_bytes, s);
  GemmArgs ga;
  ga.x = x;
  ga.w = w;
  ga.d = y;
  ga.M = M;
  ga.N = N;
  ga.K = K;
  ga.ldx = K;
  ga.ldw = K;
  ga.ldd = N;
  ga.w_mn_major = false;
  ga.elt = dtype == MLORA_DTYPE_BF16 ? Elt::kBF16 : Elt::kF16;
  ga.out_dtype = dtype;
  return launch_gemm(ga, s);
}

size_t mlora_merge_workspace_bytes(int64_t N, int64_t K, int64_t r, int dtype) {
  if (N <= 0 || K <= 0 || r <= 0) return 0;
  return merge_ws(N, K, r, dtype);
}

int mlora_merge(const void* w0, const void* a, const void* b, void* w_out, int64_t N, int64_t K,
                int64_t r, float alpha, int dtype, void* workspace, size_t workspace_bytes,
                void* stream) {
  // out_features (N) is the GEMM's row dimension here and may be ragged.
  int rc = check_shapes(8, K, 8, r, dtype);
  if (rc) return rc;
  if (N <= 0 || N > (1 << 24)) return fail(MLORA_ERR_INVALID_ARG, "N must be in [1, 2^24]");
  if (!w0 || !a || !b || !w_out) return fail(MLORA_ERR_INVALID_ARG, "NULL tensor pointer");
  if ((rc = check_ptrs16({w0, a, b, w_out, workspace}))) return rc;
  if ((rc = check_device())) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  GemmArgs ga;
  ga.M = N;
  ga.N = K;
  ga.c = w0;
  ga.ldc = K;
  ga.d = w_out;
  ga.ldd = K;
  ga.acc_scale = alpha / static_cast<float>(r);
  ga.w_mn_major = true;
  ga.out_dtype = dtype;
  if (dtype == MLORA_DTYPE_F32) {
    const size_t need = merge_ws(N, K, r, dtype);
    if (workspace == nullptr || workspace_bytes < need)
      return fail(MLORA_ERR_WORKSPACE, "fp32 merge workspace needs " + std::to_string(need) + " bytes");
    const int64_t r8 = pad8(r);
    Carve c(workspace);
    void* bs = c.take(static_cast<size_t>(N) * 3 * r8 * 2);
    void* as = c.take(static_cast<size_t>(3 * r8) * K * 2);
    if ((rc = launch_split3_cols(static_cast<const float*>(b), N, r, r, bs, r8, 3 * r8, kHHL, s)))
      return rc;
    if ((rc = launch_split3_rows(static_cast<const float*>(a), r, K, K, as, r8, kHLH, s))) return rc;
    ga.x = bs;
    ga.w = as;
    ga.K = 3 * r8;
    ga.ldx = 3 * r8;
    ga.ldw = K;
    ga.elt = Elt::kBF16;
    return launch_gemm(ga, s);
  }
  // W' = W0 + s.B.A: GEMM over the rank with W0 as the epilogue addend.
  ga.x = b;
  ga.w = a;
  ga.K = r;
  ga.ldx = r;
  ga.ldw = K;
  ga.elt = dtype == MLORA_DTYPE_BF16 ? Elt::kBF16 : Elt::kF16;
  return launch_gemm(ga, s);
}

}  // extern "C"
