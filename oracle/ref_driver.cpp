// Test infrastructure (oracle only) -- never linked into the product.
//
// Host driver that runs the reference's OWN compute shaders on the CPU, so the
// numpy restatement in oracle/lora_oracle.py and oracle/quant_oracle.py can be
// pinned against the reference itself:
//   * kernels/lora_quantized.metal  (qlora_forward_int4 :29, qlora_forward_nf4 :97,
//                                    dequant_int4 :17, dequant_nf4 :22)
//   * kernels/lora_train.metal      (lora_train_forward :27, lora_train_backward :90,
//                                    lora_optimizer_step :158)
//   * kernels/lora_kernels.metal    (LoRAConfig :12, lora_multi_adapter :440,
//                                    lora_kv_cache_update :514; cut out by
//                                    oracle/build_ref.py into
//                                    oracle/_ref/gen/lora_kernels_subset.inc)
//   * the inline MSL bodies of python/metal_lora/kernels.py
//       LORA_FORWARD_FUSED_SOURCE :41  (the live Metal forward)
//       LORA_BACKWARD_SOURCE      :249
//       LORA_ADAMW_SOURCE         :314
//       LORA_MAINTENANCE_SOURCE   :351
//     extracted at build time by oracle/build_ref.py into oracle/_ref/gen/*.inc and
//     wrapped here in functions whose parameters carry the names that
//     mx.fast.metal_kernel binds (kernels.py:377-464).
//
// The sources are included from the reference tree at build time; nothing of
// them is stored in this repository.
//
// Emulation of a Metal dispatch: every threadgroup runs on one host thread; its
// threads run one after another.  A kernel with B threadgroup barriers is run
// B+1 times over all of its threads ("passes"): pass p sees every threadgroup
// array fully written by pass p-1, so after B+1 passes each thread has observed
// the same values it would on the GPU.  Outputs written with plain stores are
// idempotent across passes; atomics only take effect in the final pass.  In-place
// read-modify-write kernels (AdamW, maintenance, optimizer step) have no barrier
// and run exactly once.
#include <metal_stdlib>
#include <cstring>

thread_local bool msl_emul_final_pass = true;

#include "lora_quantized.metal"
#include "lora_train.metal"
#include "lora_kernels_subset.inc"

namespace mlx_inline {
typedef float T;  // mx.fast.metal_kernel template T = x.dtype; pinned in float32

// kernels.py:41-144 (input_names / output_names from kernels.py:395-405)
static void lora_forward_fused(const T* x, const T* W0, const T* A, const T* B,
                               const uint* const_batch_size, const uint* const_seq_len,
                               const uint* const_in_features, const uint* const_out_features,
                               const uint* const_rank, const float* const_alpha, T* out,
                               uint3 thread_position_in_grid, uint3 threadgroup_position_in_grid) {
#include "lora_forward_fused.inc"
}

// kernels.py:249-308 (input_names from kernels.py:431-441); grad_A/grad_B are
// updated in place through atomic casts, exactly as written there.
static void lora_backward_fused(const T* grad_output, const T* x, const T* A, const T* B,
                                const float* grad_A, const float* grad_B,
                                const uint* const_batch_size, const uint* const_seq_len,
                                const uint* const_in_features, const uint* const_out_features,
                                const uint* const_rank, const float* const_alpha,
                                const float* const_clip, uint3 thread_position_in_grid,
                                uint3 threadgroup_position_in_grid) {
#include "lora_backward_fused.inc"
}

// kernels.py:314-344 (input_names from kernels.py:452-459).  The body stores
// into param/grad/m/v, so they are declared writable here (MLX binds inputs
// as const device pointers, under which this body would not compile).
static void lora_adamw_step(T* param, float* grad, float* m, float* v, const float* gpu_state,
                            const uint* const_size, const float* const_lr,
                            const float* const_beta1, const float* const_beta2,
                            const float* const_eps, const float* const_wd,
                            uint3 thread_position_in_grid) {
#include "lora_adamw_step.inc"
}

// kernels.py:351-362 (input_names from kernels.py:380-383)
static void lora_maintenance(float* gpu_state, const float* beta1, const float* beta2,
                             uint3 thread_position_in_grid) {
#include "lora_maintenance.inc"
}
}  // namespace mlx_inline

// Runs a (gx, gy, gz) grid of threadgroups with `tg` threads each.
template <class F>
static void run_grid(uint gx, uint gy, uint gz, uint tg, int passes, F&& fn) {
  const long n = (long)gx * gy * gz;
#pragma omp parallel for schedule(dynamic)
  for (long g = 0; g < n; ++g) {
    uint3 tgid{(uint)(g % gx), (uint)((g / gx) % gy), (uint)(g / ((long)gx * gy))};
    for (int p = 0; p < passes; ++p) {
      msl_emul_final_pass = (p == passes - 1);
      for (uint lid = 0; lid < tg; ++lid) fn(tgid, lid);
    }
  }
  msl_emul_final_pass = true;
}

// Serial variant for kernels whose atomics must not race across host threads.
template <class F>
static void run_grid_serial(uint gx, uint gy, uint gz, uint tg, int passes, F&& fn) {
  for (uint z = 0; z < gz; ++z)
    for (uint y = 0; y < gy; ++y)
      for (uint x = 0; x < gx; ++x) {
        uint3 tgid{x, y, z};
        for (int p = 0; p < passes; ++p) {
          msl_emul_final_pass = (p == passes - 1);
          for (uint lid = 0; lid < tg; ++lid) fn(tgid, lid);
        }
      }
  msl_emul_final_pass = true;
}

extern "C" {

// ---- inline kernels of python/metal_lora/kernels.py --------------------------

// Dispatch of kernels.py:546-561: grid (ceil(D/256)*256, S, B), threadgroup 256.
void mlref_lora_forward_fused(const float* x, const float* W0, const float* A, const float* B,
                              float* out, uint batch, uint seq, uint K, uint D, uint R,
                              float alpha) {
  const uint ntg = (D + 255) / 256;
  run_grid(ntg, seq, batch, 256, 3, [&](uint3 tgid, uint lid) {
    uint3 tpig{tgid.x * 256 + lid, tgid.y, tgid.z};
    mlx_inline::lora_forward_fused(x, W0, A, B, &batch, &seq, &K, &D, &R, &alpha, out, tpig, tgid);
  });
}

// Dispatch of kernels.py:597-611: grid (1, S, B) threadgroups of 256.  grad_A
// [R*K] and grad_B [D*R] must be zeroed by the caller (kernels.py:586-587).
void mlref_lora_backward_fused(const float* grad_output, const float* x, const float* A,
                               const float* B, float* grad_A, float* grad_B, uint batch,
                               uint seq, uint K, uint D, uint R, float alpha, float clip) {
  run_grid_serial(1, seq, batch, 256, 3, [&](uint3 tgid, uint lid) {
    uint3 tpig{tgid.x * 256 + lid, tgid.y, tgid.z};
    mlx_inline::lora_backward_fused(grad_output, x, A, B, grad_A, grad_B, &batch, &seq, &K, &D,
                                    &R, &alpha, &clip, tpig, tgid);
  });
}

// Dispatch of kernels.py:630-643: one thread per element.  gpu_state = [step, b1^t, b2^t].
void mlref_lora_adamw_step(float* param, float* grad, float* m, float* v, const float* gpu_state,
                           uint size, float lr, float b1, float b2, float eps, float wd) {
  const uint ntg = (size + 255) / 256;
  run_grid(ntg, 1, 1, 256, 1, [&](uint3 tgid, uint lid) {
    uint3 tpig{tgid.x * 256 + lid, 0, 0};
    mlx_inline::lora_adamw_step(param, grad, m, v, gpu_state, &size, &lr, &b1, &b2, &eps, &wd,
                                tpig);
  });
}

// kernels.py:484-499: a single thread.
void mlref_lora_maintenance(float* gpu_state, float b1, float b2) {
  mlx_inline::lora_maintenance(gpu_state, &b1, &b2, uint3{0, 0, 0});
}

// ---- kernels/lora_quantized.metal ------------------------------------------

float mlref_dequant_nf4(uchar packed, int high_nibble, float absmax) {
  return dequant_nf4(packed, high_nibble != 0, absmax);
}

float mlref_dequant_int4(uchar packed, int high_nibble, float scale, float zero_point) {
  return dequant_int4(packed, high_nibble != 0, scale, zero_point);
}

// Grid (ceil(D/256), S, B) x 256 threads, as the shader's indexing implies.
void mlref_qlora_forward_nf4(const uchar* W0_quant, const float* W0_absmax, const uint16_t* x,
                             const uint16_t* A, const uint16_t* B, uint16_t* out, uint batch,
                             uint seq, uint K, uint D, uint R, float alpha, uint block_size) {
  const uint ntg = (D + 255) / 256;
  run_grid(ntg, seq, batch, 256, 2, [&](uint3 tgid, uint lid) {
    qlora_forward_nf4(W0_quant, W0_absmax, (const half*)x, (const half*)A, (const half*)B,
                      (half*)out, batch, seq, K, D, R, alpha, block_size, tgid, lid);
  });
}

void mlref_qlora_forward_int4(const uchar* W0_quant, const float* W0_scales,
                              const float* W0_zeros, const uint16_t* x, const uint16_t* A,
                              const uint16_t* B, uint16_t* out, uint batch, uint seq, uint K,
                              uint D, uint R, float alpha) {
  const uint ntg = (D + 255) / 256;
  run_grid(ntg, seq, batch, 256, 2, [&](uint3 tgid, uint lid) {
    qlora_forward_int4(W0_quant, W0_scales, W0_zeros, (const half*)x, (const half*)A,
                       (const half*)B, (half*)out, batch, seq, K, D, R, alpha, tgid, lid);
  });
}

// ---- kernels/lora_train.metal -------------------------------------------------

static TrainConfig make_cfg(uint batch, uint seq, uint K, uint D, uint R, float alpha,
                            float clip) {
  TrainConfig c;
  std::memset(&c, 0, sizeof(c));
  c.batch_size = batch;
  c.seq_len = seq;
  c.in_features = K;
  c.out_features = D;
  c.rank = R;
  c.alpha = alpha;
  c.grad_clip = clip;
  c.accumulation_steps = 1;
  return c;
}

void mlref_train_forward(const uint16_t* x, const uint16_t* W0, const uint16_t* A,
                         const uint16_t* B, uint16_t* out, float* Ax_cache, uint batch, uint seq,
                         uint K, uint D, uint R, float alpha) {
  TrainConfig cfg = make_cfg(batch, seq, K, D, R, alpha, 0.f);
  const uint ntg = (D + 255) / 256;
  run_grid(ntg, seq, batch, 256, 3, [&](uint3 tgid, uint lid) {
    lora_train_forward((const half*)x, (const half*)W0, (const half*)A, (const half*)B,
                       (half*)out, Ax_cache, cfg, tgid, lid);
  });
}

void mlref_train_backward(const uint16_t* grad_output, const uint16_t* x, const float* Ax_cache,
                          const uint16_t* A, const uint16_t* B, float* grad_A, float* grad_B,
                          uint batch, uint seq, uint K, uint D, uint R, float alpha, float clip) {
  TrainConfig cfg = make_cfg(batch, seq, K, D, R, alpha, clip);
  run_grid_serial(1, seq, batch, 256, 3, [&](uint3 tgid, uint lid) {
    lora_train_backward((const half*)grad_output, (const half*)x, Ax_cache, (const half*)A,
                        (const half*)B, grad_A, grad_B, cfg, tgid, lid);
  });
}

void mlref_optimizer_step(uint16_t* A, uint16_t* B, float* grad_A, float* grad_B, float* m_A,
                          float* v_A, float* m_B, float* v_B, float lr, float b1, float b2,
                          float eps, float wd, uint step, uint A_size, uint B_size,
                          uint accum_steps) {
  const uint total = A_size + B_size;
  for (uint tid = 0; tid < total; ++tid)
    lora_optimizer_step((half*)A, (half*)B, grad_A, grad_B, m_A, v_A, m_B, v_B, lr, b1, b2, eps,
                        wd, step, A_size, B_size, accum_steps, tid);
}

// ---- kernels/lora_kernels.metal ------------------------------------------------

// lora_multi_adapter :440-508: one threadgroup of 256 per (256 outputs, token,
// sample); two barriers -> three passes.  fp32 throughout.
void mlref_multi_adapter(const float* x, const float* W0, const float* adapters_A,
                         const float* adapters_B, const uint* adapter_ids, float* out, uint batch,
                         uint seq, uint K, uint D, uint R, uint num_adapters, float alpha) {
  LoRAConfig cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.batch_size = batch;
  cfg.seq_len = seq;
  cfg.in_features = K;
  cfg.out_features = D;
  cfg.rank = R;
  cfg.alpha = alpha;
  run_grid((D + 255) / 256, seq, batch, 256, 3, [&](uint3 tgid, uint lid) {
    lora_multi_adapter(x, W0, adapters_A, adapters_B, adapter_ids, out, cfg, num_adapters, tgid,
                       lid);
  });
}

// lora_kv_cache_update :514-586: one new token per sequence; the caches are
// [batch, 8192, D] half (the shader's fixed max_seq); two barriers -> three passes.
void mlref_kv_cache_update(const uint16_t* x, const uint16_t* W_K, const uint16_t* W_V,
                           const uint16_t* A_K, const uint16_t* B_K, const uint16_t* A_V,
                           const uint16_t* B_V, uint16_t* K_cache, uint16_t* V_cache, uint batch,
                           uint cur_pos, uint D, uint R, float alpha) {
  run_grid((D + 255) / 256, 1, batch, 256, 3, [&](uint3 tgid, uint lid) {
    lora_kv_cache_update((const half*)x, (const half*)W_K, (const half*)W_V, (const half*)A_K,
                         (const half*)B_K, (const half*)A_V, (const half*)B_V, (half*)K_cache,
                         (half*)V_cache, batch, cur_pos, D, R, alpha, tgid, lid);
  });
}

}  // extern "C"
