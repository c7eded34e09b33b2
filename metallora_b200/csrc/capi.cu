// C-ABI layer: argument validation, workspace planning, tensor-map encoding and
// the launch sequences of the LoRA-linear operations.  See
// include/metallora_b200.h for the contract of each entry point.
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

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

int check_shapes(int64_t M, int64_t K, int64_t N, int64_t r, int dtype) {
  if (M <= 0 || K <= 0 || N <= 0) return fail(MLORA_ERR_INVALID_ARG, "M, K, N must be positive");
  if (r < 1 || r > 256) return fail(MLORA_ERR_INVALID_ARG, "rank must be in [1, 256]");
  if (dtype != MLORA_DTYPE_BF16 && dtype != MLORA_DTYPE_F16)
    return fail(MLORA_ERR_UNSUPPORTED, "dtype must be BF16 or F16");
  if (K % 8 || N % 8 || r % 8)
    return fail(MLORA_ERR_UNSUPPORTED, "K, N and r must be multiples of 8 (16-byte rows)");
  if (M > (int64_t(1) << 31) - 1 || K > (1 << 24) || N > (1 << 24))
    return fail(MLORA_ERR_UNSUPPORTED, "shape too large");
  return MLORA_OK;
}

// ---- forward plan --------------------------------------------------------
struct FwdPlan {
  int64_t R, R64;
  int splits;
  uint32_t* counters;
  void* xa_rows;
  void* xa_t;
  float* partials;
  size_t bytes;
};

FwdPlan plan_forward(void* ws, int64_t M, int64_t K, int64_t r, bool need_xa_t) {
  FwdPlan p;
  p.R = rank_tile(r);
  p.R64 = pad64(p.R);
  p.splits = rank_splits(M, K);
  Carve c(ws);
  p.counters = static_cast<uint32_t*>(c.take(((M + 127) / 128) * 4));
  p.xa_rows = c.take(static_cast<size_t>(M) * p.R64 * 2);
  p.xa_t = need_xa_t ? c.take(static_cast<size_t>(p.R) * pad8(M) * 2) : nullptr;
  p.partials = p.splits > 1 ? static_cast<float*>(c.take(size_t(p.splits) * M * p.R * 4)) : nullptr;
  p.bytes = align_up(c.off, 256);
  return p;
}

// ---- backward plan -------------------------------------------------------
struct BwdPlan {
  int64_t R, R64;
  int rsplits, wsplits;
  uint32_t* counters;  // [tiles_m] rank(U) | [tiles_m] rank(T) | [N/128] dB | [K/128] dA
  size_t counter_bytes;
  void* bt;
  void* u_rows;
  void* u_t;
  void* xa_t;
  float* rpartials;
  float* wpart_db;
  float* wpart_da;
  size_t bytes;
};

BwdPlan plan_backward(void* ws, int64_t M, int64_t K, int64_t N, int64_t r, bool need_xa_t) {
  BwdPlan p;
  p.R = rank_tile(r);
  p.R64 = pad64(p.R);
  p.rsplits = rank_splits(M, N > K ? N : K);
  p.wsplits = wgrad_splits(M, N > K ? N : K, 2);
  const int64_t tm = (M + 127) / 128, tn = (N + 127) / 128, tk = (K + 127) / 128;
  Carve c(ws);
  p.counter_bytes = static_cast<size_t>(2 * tm + tn + tk) * 4;
  p.counters = static_cast<uint32_t*>(c.take(p.counter_bytes));
  p.bt = c.take(static_cast<size_t>(p.R) * N * 2);
  p.u_rows = c.take(static_cast<size_t>(M) * p.R64 * 2);
  p.u_t = c.take(static_cast<size_t>(p.R) * pad8(M) * 2);
  p.xa_t = need_xa_t ? c.take(static_cast<size_t>(p.R) * pad8(M) * 2) : nullptr;
  p.rpartials = p.rsplits > 1 ? static_cast<float*>(c.take(size_t(p.rsplits) * M * p.R * 4)) : nullptr;
  p.wpart_db = p.wsplits > 1 ? static_cast<float*>(c.take(size_t(p.wsplits) * N * p.R * 4)) : nullptr;
  p.wpart_da = p.wsplits > 1 ? static_cast<float*>(c.take(size_t(p.wsplits) * K * p.R * 4)) : nullptr;
  p.bytes = align_up(c.off, 256);
  return p;
}

}  // namespace

void set_error(const std::string& msg) { t_last_error = msg; }

bool make_tmap_2d_16b(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled entry point unavailable");
    return false;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
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

size_t mlora_lora_forward_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r) {
  (void)N;
  if (M <= 0 || K <= 0 || r <= 0) return 0;
  return plan_forward(nullptr, M, K, r, true).bytes;
}

int mlora_lora_forward(const void* x, const void* w0, const void* a, const void* b, void* y,
                       void* saved_xa, int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                       int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_shapes(M, K, N, r, dtype);
  if (rc) return rc;
  if (!x || !w0 || !a || !b || !y) return fail(MLORA_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(x) || !aligned16(w0) || !aligned16(a) || !aligned16(b) || !aligned16(y) ||
      (saved_xa && !aligned16(saved_xa)))
    return fail(MLORA_ERR_INVALID_ARG, "tensor pointers must be 16-byte aligned");
  if ((rc = check_device())) return rc;
  const FwdPlan need = plan_forward(nullptr, M, K, r, saved_xa == nullptr);
  if (workspace == nullptr || workspace_bytes < need.bytes || !aligned16(workspace))
    return fail(MLORA_ERR_WORKSPACE, "forward workspace needs " + std::to_string(need.bytes) + " bytes");
  const FwdPlan p = plan_forward(workspace, M, K, r, saved_xa == nullptr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const Elt elt = dtype == MLORA_DTYPE_BF16 ? Elt::kBF16 : Elt::kF16;

  cudaError_t e = cudaMemsetAsync(p.counters, 0, ((M + 127) / 128) * 4, s);
  if (e != cudaSuccess) return fail(MLORA_ERR_CUDA, std::string("memset: ") + cudaGetErrorString(e));

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
  ra.partials = p.partials;
  ra.counters = p.counters;
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
  ga.ldd = N;
  ga.w_mn_major = false;
  ga.elt = elt;
  ga.out_dtype = dtype;
  return launch_gemm(ga, s);
}

size_t mlora_lora_backward_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r) {
  if (M <= 0 || K <= 0 || N <= 0 || r <= 0) return 0;
  return plan_backward(nullptr, M, K, N, r, true).bytes;
}

int mlora_lora_backward(const void* dy, const void* x, const void* w0, const void* a,
                        const void* b, const void* saved_xa, void* dx, float* da, float* db,
                        int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                        float clip_value, int dtype, void* workspace, size_t workspace_bytes,
                        void* stream) {
  int rc = check_shapes(M, K, N, r, dtype);
  if (rc) return rc;
  if (!dy || !x || !a || !b || !da || !db) return fail(MLORA_ERR_INVALID_ARG, "NULL tensor pointer");
  if ((dx == nullptr) != (w0 == nullptr))
    return fail(MLORA_ERR_INVALID_ARG, "w0 and dx must be both set or both NULL");
  const void* ptrs[] = {dy, x, w0, a, b, saved_xa, dx, da, db};
  for (const void* q : ptrs)
    if (q && !aligned16(q)) return fail(MLORA_ERR_INVALID_ARG, "tensor pointers must be 16-byte aligned");
  if ((rc = check_device())) return rc;
  const BwdPlan need = plan_backward(nullptr, M, K, N, r, saved_xa == nullptr);
  if (workspace == nullptr || workspace_bytes < need.bytes || !aligned16(workspace))
    return fail(MLORA_ERR_WORKSPACE, "backward workspace needs " + std::to_string(need.bytes) + " bytes");
  const BwdPlan p = plan_backward(workspace, M, K, N, r, saved_xa == nullptr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const Elt elt = dtype == MLORA_DTYPE_BF16 ? Elt::kBF16 : Elt::kF16;
  const int64_t tm = (M + 127) / 128, tn = (N + 127) / 128;
  const float scale = alpha / static_cast<float>(r);

  cudaError_t e = cudaMemsetAsync(p.counters, 0, p.counter_bytes, s);
  if (e != cudaSuccess) return fail(MLORA_ERR_CUDA, std::string("memset: ") + cudaGetErrorString(e));

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
  ra.partials = p.rpartials;
  ra.counters = p.counters;
  ra.splits = rank_splits(M, N);
  ra.elt = elt;
  if (ra.splits > p.rsplits) ra.splits = p.rsplits;
  if ((rc = launch_rank(ra, s))) return rc;

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
    rt.counters = p.counters + tm;
    rt.splits = rank_splits(M, K);
    if (rt.splits > p.rsplits) rt.splits = p.rsplits;
    if ((rc = launch_rank(rt, s))) return rc;
    xa_t = p.xa_t;
  }

  if (dx != nullptr) {
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
    if ((rc = launch_gemm(ga, s))) return rc;
  }

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
  w[0].clip = clip_value;
  w[0].partials = p.wpart_db;
  w[0].counters = p.counters + 2 * tm;
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
  w[1].partials = p.wpart_da;
  w[1].counters = p.counters + 2 * tm + tn;
  return launch_wgrad(w, 2, s);
}

}  // extern "C"
