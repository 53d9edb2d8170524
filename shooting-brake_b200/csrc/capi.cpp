// C-ABI implementation (include/sbb200.h): argument validation, workspace
// planning and the kernel-choice driver for the routed-expert NVFP4 MoE.
//
// Host C++ only; exceptions never cross the ABI (the reference's rule,
// src/phase1/b70_provider.cpp:1825-1848). Errors are reported as int status
// plus a per-thread (stateless op) or per-provider (provider) message.
#include "sbb200.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <unordered_map>

#include "kernels.h"
#include "moe_driver.h"

namespace {

thread_local std::string t_last_error;

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(SBB200_ECUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

bool dtype_ok(int dt) { return dt == SBB200_F32 || dt == SBB200_F16 || dt == SBB200_BF16; }

}  // namespace

namespace sbb {

void set_last_error(const std::string& msg) { t_last_error = msg; }

int validate_shape(size_t M, size_t E, size_t top_k, size_t K, size_t I, int act_dt, int out_dt,
                   std::string* why) {
  if (M == 0 || E == 0 || top_k == 0 || K == 0 || I == 0) {
    *why = "NVFP4 MoE dimensions must be nonzero";
    return SBB200_EINVAL;
  }
  if (K % 32 != 0 || I % 32 != 0) {
    *why = "NVFP4 MoE K/I must be multiples of 32";
    return SBB200_EINVAL;
  }
  if (!dtype_ok(act_dt) || !dtype_ok(out_dt)) {
    *why = "activation and output dtypes must be f32, f16 or bf16";
    return SBB200_EINVAL;
  }
  if (E > (size_t)kMaxExperts) {
    *why = "E above the supported maximum of " + std::to_string(kMaxExperts);
    return SBB200_EUNSUPPORTED;
  }
  if (top_k > (size_t)kMaxTopK) {
    *why = "top_k above the supported maximum of " + std::to_string(kMaxTopK);
    return SBB200_EUNSUPPORTED;
  }
  if (M > (size_t)0x7fffffff / top_k || K > 65536 || I > 65536) {
    *why = "shape exceeds 32-bit route indexing";
    return SBB200_EUNSUPPORTED;
  }
  return SBB200_OK;
}

}  // namespace sbb

extern "C" {

size_t sbb200_abi_version(void) { return SBB200_ABI_VERSION; }

size_t sbb200_last_error(char* buf, size_t size) {
  const size_t need = t_last_error.size() + 1;
  if (buf && size) {
    const size_t n = need <= size ? need - 1 : size - 1;
    std::memcpy(buf, t_last_error.data(), n);
    buf[n] = '\0';
  }
  return need;
}

size_t sbb200_nvfp4_moe_workspace_bytes(size_t M, size_t E, size_t top_k, size_t K, size_t I,
                                        int act_dt) {
  (void)act_dt;
  return sbb::plan_workspace(M, E, top_k, K, I).total;
}

int sbb200_nvfp4_moe_launches(size_t M, size_t E, size_t top_k, size_t K, size_t I,
                              int act_dt) {
  (void)E;
  (void)act_dt;
  return sbb::count_launches(static_cast<int64_t>(M), static_cast<int>(top_k),
                             static_cast<int>(K), static_cast<int>(I));
}

int sbb200_nvfp4_moe(void* stream, const void* hidden, const int32_t* topk_ids,
                     const float* topk_weights, const void* w13, const void* w13_scales,
                     const float* w13_global_scales, const void* w2, const void* w2_scales,
                     const float* w2_global_scales, void* workspace, size_t workspace_bytes,
                     void* out, int out_dt, size_t M, size_t E, size_t top_k, size_t K,
                     size_t I, int act_dt, int multiply_router_weight) {
  return sbb200_nvfp4_moe_staged(stream, hidden, topk_ids, topk_weights, w13, w13_scales,
                                 w13_global_scales, w2, w2_scales, w2_global_scales, workspace,
                                 workspace_bytes, out, out_dt, M, E, top_k, K, I, act_dt,
                                 multiply_router_weight, nullptr, SBB200_STAGE_EVENTS);
}

int sbb200_nvfp4_moe_staged(void* stream, const void* hidden, const int32_t* topk_ids,
                            const float* topk_weights, const void* w13, const void* w13_scales,
                            const float* w13_global_scales, const void* w2, const void* w2_scales,
                            const float* w2_global_scales, void* workspace,
                            size_t workspace_bytes, void* out, int out_dt, size_t M, size_t E,
                            size_t top_k, size_t K, size_t I, int act_dt,
                            int multiply_router_weight, void* const* stage_events,
                            size_t n_stage_events) {
  try {
    if (stage_events && n_stage_events != SBB200_STAGE_EVENTS)
      return fail(SBB200_EINVAL, "stage_events must hold SBB200_STAGE_EVENTS entries");
    std::string why;
    int rc = sbb::validate_shape(M, E, top_k, K, I, act_dt, out_dt, &why);
    if (rc != SBB200_OK) return fail(rc, why);
    if (!hidden || !topk_ids || !w13 || !w13_scales || !w13_global_scales || !w2 ||
        !w2_scales || !w2_global_scales || !workspace || !out ||
        (multiply_router_weight && !topk_weights)) {
      return fail(SBB200_EINVAL, "nvfp4_moe received a null pointer");
    }
    const sbb::WorkspacePlan plan = sbb::plan_workspace(M, E, top_k, K, I);
    if (workspace_bytes < plan.total) {
      return fail(SBB200_EWORKSPACE, "workspace holds " + std::to_string(workspace_bytes) +
                                         " bytes, the call needs " + std::to_string(plan.total));
    }
    sbb::MoeArgs a{};
    a.hidden = hidden;
    a.act_dt = act_dt;
    a.ids = topk_ids;
    a.weights = topk_weights;
    a.multiply_router_weight = multiply_router_weight;
    a.w13 = static_cast<const uint8_t*>(w13);
    a.s13 = static_cast<const uint8_t*>(w13_scales);
    a.g13 = w13_global_scales;
    a.w2 = static_cast<const uint8_t*>(w2);
    a.s2 = static_cast<const uint8_t*>(w2_scales);
    a.g2 = w2_global_scales;
    a.out = out;
    a.out_dt = out_dt;
    a.M = (int64_t)M;
    a.E = (int)E;
    a.top_k = (int)top_k;
    a.K = (int)K;
    a.I = (int)I;
    a.stage_events = stage_events;
    cudaError_t err = sbb::run_moe(a, plan, workspace, static_cast<cudaStream_t>(stream), &why);
    if (err != cudaSuccess) return fail(SBB200_ECUDA, why + ": " + cudaGetErrorString(err));
    return SBB200_OK;
  } catch (const std::exception& e) {
    return fail(SBB200_ECUDA, std::string("nvfp4_moe: ") + e.what());
  } catch (...) {
    return fail(SBB200_ECUDA, "nvfp4_moe: unknown exception");
  }
}

int sbb200_nvfp4_moe_w4a4(void* stream, const void* hidden, const int32_t* topk_ids,
                          const float* topk_weights, const void* w13, const void* w13_scales,
                          const float* w13_global_scales, const void* w2, const void* w2_scales,
                          const float* w2_global_scales, const float* a13_gscale,
                          const float* a2_gscale, const float* alpha13, const float* alpha2,
                          void* workspace, size_t workspace_bytes, void* out, int out_dt,
                          size_t M, size_t E, size_t top_k, size_t K, size_t I, int act_dt,
                          int multiply_router_weight, void* const* stage_events,
                          size_t n_stage_events) {
  try {
    if (stage_events && n_stage_events != SBB200_STAGE_EVENTS)
      return fail(SBB200_EINVAL, "stage_events must hold SBB200_STAGE_EVENTS entries");
    std::string why;
    int rc = sbb::validate_shape(M, E, top_k, K, I, act_dt, out_dt, &why);
    if (rc != SBB200_OK) return fail(rc, why);
    const bool stat = a13_gscale || a2_gscale || alpha13 || alpha2;
    if (stat && !(a13_gscale && a2_gscale && alpha13 && alpha2))
      return fail(SBB200_EINVAL, "nvfp4_moe_w4a4: static scales need a13_gscale, a2_gscale, "
                                 "alpha13 and alpha2 together");
    if (!hidden || !topk_ids || !w13 || !w13_scales || !w2 || !w2_scales || !workspace || !out ||
        (!stat && (!w13_global_scales || !w2_global_scales)) ||
        (multiply_router_weight && !topk_weights))
      return fail(SBB200_EINVAL, "nvfp4_moe_w4a4 received a null pointer");
    if (!sbb::bs_supported((int)K, (int)I))
      return fail(SBB200_EUNSUPPORTED, "nvfp4_moe_w4a4 needs K and I multiples of 256");
    const sbb::WorkspacePlan plan = sbb::plan_workspace(M, E, top_k, K, I);
    if (workspace_bytes < plan.total)
      return fail(SBB200_EWORKSPACE, "workspace holds " + std::to_string(workspace_bytes) +
                                         " bytes, the call needs " + std::to_string(plan.total));
    sbb::MoeArgs a{};
    a.hidden = hidden;
    a.act_dt = act_dt;
    a.ids = topk_ids;
    a.weights = topk_weights;
    a.multiply_router_weight = multiply_router_weight;
    a.w13 = static_cast<const uint8_t*>(w13);
    a.s13 = static_cast<const uint8_t*>(w13_scales);
    a.g13 = w13_global_scales;
    a.w2 = static_cast<const uint8_t*>(w2);
    a.s2 = static_cast<const uint8_t*>(w2_scales);
    a.g2 = w2_global_scales;
    a.out = out;
    a.out_dt = out_dt;
    a.M = (int64_t)M;
    a.E = (int)E;
    a.top_k = (int)top_k;
    a.K = (int)K;
    a.I = (int)I;
    a.act_terms = 1;
    a.a13_gscale = a13_gscale;
    a.a2_gscale = a2_gscale;
    a.alpha13 = alpha13;
    a.alpha2 = alpha2;
    a.stage_events = stage_events;
    cudaError_t err = sbb::run_moe(a, plan, workspace, static_cast<cudaStream_t>(stream), &why);
    if (err != cudaSuccess) return fail(SBB200_ECUDA, why + ": " + cudaGetErrorString(err));
    return SBB200_OK;
  } catch (...) {
    return fail(SBB200_ECUDA, "nvfp4_moe_w4a4: host exception");
  }
}

int sbb200_router_topk(void* stream, const void* router_logits, int dt, size_t M, size_t E,
                       size_t top_k, int32_t* topk_ids, float* topk_weights) {
  if (!dtype_ok(dt)) return fail(SBB200_EINVAL, "router logits dtype must be f32, f16 or bf16");
  if (E == 0 || E > (size_t)sbb::kMaxExperts || top_k == 0 || top_k > E ||
      top_k > (size_t)sbb::kMaxTopK)
    return fail(SBB200_EINVAL, "router top-k needs 1 <= top_k <= min(E, 64) and E <= 512");
  if (M == 0) return SBB200_OK;
  if (!router_logits || !topk_ids || !topk_weights)
    return fail(SBB200_EINVAL, "router top-k received a null pointer");
  const cudaError_t err = sbb::launch_router_topk(router_logits, dt, (int64_t)M, (int)E,
                                                  (int)top_k, topk_ids, topk_weights,
                                                  static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "router top-k");
  return SBB200_OK;
}

int sbb200_nvfp4_moe_from_logits(void* stream, const void* hidden, const void* router_logits,
                                 int logits_dt, int32_t* topk_ids, float* topk_weights,
                                 const void* w13, const void* w13_scales,
                                 const float* w13_global_scales, const void* w2,
                                 const void* w2_scales, const float* w2_global_scales,
                                 void* workspace, size_t workspace_bytes, void* out, int out_dt,
                                 size_t M, size_t E, size_t top_k, size_t K, size_t I,
                                 int act_dt, int multiply_router_weight) {
  try {
    std::string why;
    int rc = sbb::validate_shape(M, E, top_k, K, I, act_dt, out_dt, &why);
    if (rc != SBB200_OK) return fail(rc, why);
    if (!dtype_ok(logits_dt)) return fail(SBB200_EINVAL, "router logits dtype must be f32, f16 or bf16");
    if (top_k > E) return fail(SBB200_EINVAL, "router top-k needs top_k <= E");
    if (!hidden || !router_logits || !topk_ids || !topk_weights || !w13 || !w13_scales ||
        !w13_global_scales || !w2 || !w2_scales || !w2_global_scales || !workspace || !out)
      return fail(SBB200_EINVAL, "nvfp4_moe_from_logits received a null pointer");
    const sbb::WorkspacePlan plan = sbb::plan_workspace(M, E, top_k, K, I);
    if (workspace_bytes < plan.total)
      return fail(SBB200_EWORKSPACE, "workspace holds " + std::to_string(workspace_bytes) +
                                         " bytes, the call needs " + std::to_string(plan.total));
    sbb::MoeArgs a{};
    a.hidden = hidden;
    a.act_dt = act_dt;
    a.ids = topk_ids;
    a.weights = topk_weights;
    a.router_logits = router_logits;
    a.logits_dt = logits_dt;
    a.routed_ids = topk_ids;
    a.routed_weights = topk_weights;
    a.multiply_router_weight = multiply_router_weight;
    a.w13 = static_cast<const uint8_t*>(w13);
    a.s13 = static_cast<const uint8_t*>(w13_scales);
    a.g13 = w13_global_scales;
    a.w2 = static_cast<const uint8_t*>(w2);
    a.s2 = static_cast<const uint8_t*>(w2_scales);
    a.g2 = w2_global_scales;
    a.out = out;
    a.out_dt = out_dt;
    a.M = (int64_t)M;
    a.E = (int)E;
    a.top_k = (int)top_k;
    a.K = (int)K;
    a.I = (int)I;
    cudaError_t err = sbb::run_moe(a, plan, workspace, static_cast<cudaStream_t>(stream), &why);
    if (err != cudaSuccess) return fail(SBB200_ECUDA, why + ": " + cudaGetErrorString(err));
    return SBB200_OK;
  } catch (...) {
    return fail(SBB200_ECUDA, "nvfp4_moe_from_logits: host exception");
  }
}

int sbb200_nvfp4_moe_bad_ids(void* stream, const void* workspace, uint32_t* count) {
  if (!workspace || !count) return fail(SBB200_EINVAL, "bad_ids received a null pointer");
  const uint32_t* status = reinterpret_cast<const uint32_t*>(
      static_cast<const char*>(workspace) + sbb::kStatusOffset);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err = cudaMemcpyAsync(count, status, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  if (err != cudaSuccess) return cuda_fail(err, "bad_ids");
  return SBB200_OK;
}

int sbb200_nvfp4_moe_device_errors(void* stream, const void* workspace, uint32_t* errors) {
  if (!workspace || !errors) return fail(SBB200_EINVAL, "device_errors received a null pointer");
  const uint32_t* status = reinterpret_cast<const uint32_t*>(
      static_cast<const char*>(workspace) + sbb::kStatusOffset);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err =
      cudaMemcpyAsync(errors, status + 1, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  if (err != cudaSuccess) return cuda_fail(err, "device_errors");
  return SBB200_OK;
}

uint64_t sbb200_set_kernel_wait_ns(uint64_t ns) { return sbb::set_kernel_wait_ns(ns); }

int sbb200_device_errors(void* stream, uint32_t* errors) {
  if (!errors) return fail(SBB200_EINVAL, "device_errors received a null pointer");
  const cudaError_t err = sbb::read_sticky_errors(static_cast<cudaStream_t>(stream), errors);
  if (err != cudaSuccess) return cuda_fail(err, "device_errors");
  return SBB200_OK;
}

size_t sbb200_route_plan_scratch_bytes(size_t routes, size_t E) {
  return sbb::route_plan_scratch_bytes(routes, E);
}

int sbb200_route_plan(void* stream, const int32_t* topk_ids, size_t M, size_t top_k, size_t E,
                      int32_t* counts, int32_t* offsets, int32_t* sorted, int32_t* slot_of,
                      void* scratch, uint32_t* bad_ids) {
  if (E == 0 || E > (size_t)sbb::kMaxExperts)
    return fail(SBB200_EINVAL, "route_plan: E must be in [1, 512]");
  if (top_k != 0 && M > (size_t)0x7fffffff / top_k)
    return fail(SBB200_EUNSUPPORTED, "route_plan: too many routes");
  if (!counts || !offsets || (M * top_k != 0 && (!topk_ids || !sorted || !slot_of || !scratch)))
    return fail(SBB200_EINVAL, "route_plan received a null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The status word lives at the start of the scratch when the caller gives no
  // counter of its own.
  uint32_t* status = bad_ids;
  char* sc = static_cast<char*>(scratch);
  int32_t* chunk_counts = reinterpret_cast<int32_t*>(sc + 256);
  if (!status) {
    status = reinterpret_cast<uint32_t*>(sc);
  }
  cudaError_t err = sbb::launch_route_plan(topk_ids, (int64_t)(M * top_k), (int)E, chunk_counts,
                                           counts, offsets, sorted, slot_of, status, s);
  if (err != cudaSuccess) return cuda_fail(err, "route_plan");
  return SBB200_OK;
}

int sbb200_nvfp4_dequant(void* stream, const void* q, const void* sf, const float* g,
                         size_t rows_per_scale, float* out, size_t rows, size_t cols) {
  if (!q || !sf || !g || !out || rows_per_scale == 0)
    return fail(SBB200_EINVAL, "dequant received a null pointer or zero rows_per_scale");
  if (cols % 16 != 0) return fail(SBB200_EINVAL, "dequant: cols must be a multiple of 16");
  cudaError_t err = sbb::launch_dequant(static_cast<const uint8_t*>(q),
                                        static_cast<const uint8_t*>(sf), g,
                                        (int64_t)rows_per_scale, out, (int64_t)rows,
                                        (int64_t)cols, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "dequant");
  return SBB200_OK;
}

int sbb200_nvfp4_quantize(void* stream, const void* x, int in_dt, const float* gq,
                          size_t rows_per_scale, void* q, void* sf, size_t rows, size_t cols) {
  if (!x || !gq || !q || !sf || rows_per_scale == 0)
    return fail(SBB200_EINVAL, "quantize received a null pointer or zero rows_per_scale");
  if (!dtype_ok(in_dt)) return fail(SBB200_EINVAL, "quantize: input dtype must be f32, f16 or bf16");
  if (cols % 16 != 0) return fail(SBB200_EINVAL, "quantize: cols must be a multiple of 16");
  cudaError_t err = sbb::launch_quantize(x, in_dt, gq, (int64_t)rows_per_scale,
                                         static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf),
                                         (int64_t)rows, (int64_t)cols,
                                         static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "quantize");
  return SBB200_OK;
}

// ---------------------------------------------------------------------------
// Provider
// ---------------------------------------------------------------------------

struct sbb200_provider {
  struct LayerWeights {
    size_t E;
    const uint8_t *w13, *s13, *w2, *s2;
    const float *g13, *g2;
  };
  int device = 0;
  size_t max_tokens = 0, top_k = 0, max_E = 0, K = 0, I = 0;
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  std::unordered_map<size_t, LayerWeights> layers;
  std::mutex mu;
  uint64_t generation = 1;
  uint64_t dispatches = 0;
  uint64_t allocations = 0;
  std::string last_error;

  int err(int code, const std::string& msg) {
    last_error = msg;
    t_last_error = msg;
    return code;
  }
};

sbb200_provider_t* sbb200_create(int device, size_t max_tokens, size_t top_k, size_t max_E,
                                 size_t K, size_t I) {
  try {
    std::string why;
    if (max_tokens == 0 ||
        sbb::validate_shape(max_tokens, max_E, top_k, K, I, SBB200_BF16, SBB200_F32, &why) != 0) {
      t_last_error = "create: " + (why.empty() ? std::string("max_tokens must be nonzero") : why);
      return nullptr;
    }
    auto* p = new (std::nothrow) sbb200_provider();
    if (!p) return nullptr;
    p->device = device;
    p->max_tokens = max_tokens;
    p->top_k = top_k;
    p->max_E = max_E;
    p->K = K;
    p->I = I;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) {
      p->workspace_bytes = sbb::plan_workspace(max_tokens, max_E, top_k, K, I).total;
      e = cudaMalloc(&p->workspace, p->workspace_bytes);
      if (e == cudaSuccess) ++p->allocations;
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
      t_last_error = std::string("create: ") + cudaGetErrorString(e);
      delete p;
      return nullptr;
    }
    return p;
  } catch (...) {
    t_last_error = "create: unknown exception";
    return nullptr;
  }
}

void sbb200_destroy(sbb200_provider_t* p) {
  if (!p) return;
  if (p->workspace) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    cudaFree(p->workspace);
    cudaSetDevice(prev);
  }
  delete p;
}

int sbb200_register_layer(sbb200_provider_t* p, size_t layer, size_t E, const void* w13,
                          const void* w13_scales, const float* w13_global_scales,
                          const void* w2, const void* w2_scales,
                          const float* w2_global_scales) {
  if (!p) return fail(SBB200_EINVAL, "register_layer: null provider");
  std::lock_guard<std::mutex> lock(p->mu);
  if (E == 0 || E > p->max_E)
    return p->err(SBB200_EINVAL, "register_layer: E outside [1, max_E]");
  if (!w13 || !w13_scales || !w13_global_scales || !w2 || !w2_scales || !w2_global_scales)
    return p->err(SBB200_EINVAL, "register_layer received a null pointer");
  p->layers[layer] = {E,
                      static_cast<const uint8_t*>(w13),
                      static_cast<const uint8_t*>(w13_scales),
                      static_cast<const uint8_t*>(w2),
                      static_cast<const uint8_t*>(w2_scales),
                      w13_global_scales,
                      w2_global_scales};
  ++p->generation;
  return SBB200_OK;
}

int sbb200_moe_forward(sbb200_provider_t* p, size_t layer, void* stream, const void* hidden,
                       int act_dt, const int32_t* topk_ids, const float* topk_weights,
                       void* out, int out_dt, size_t M, int multiply_router_weight) {
  if (!p) return fail(SBB200_EINVAL, "moe_forward: null provider");
  std::lock_guard<std::mutex> lock(p->mu);
  auto it = p->layers.find(layer);
  if (it == p->layers.end()) return p->err(SBB200_ENOTLOADED, "moe_forward: layer not registered");
  if (M == 0 || M > p->max_tokens)
    return p->err(SBB200_EINVAL, "moe_forward: M outside [1, max_tokens]");
  const auto& L = it->second;
  const int rc = sbb200_nvfp4_moe(stream, hidden, topk_ids, topk_weights, L.w13, L.s13, L.g13,
                                  L.w2, L.s2, L.g2, p->workspace, p->workspace_bytes, out, out_dt,
                                  M, L.E, p->top_k, p->K, p->I, act_dt, multiply_router_weight);
  if (rc != SBB200_OK) {
    p->last_error = t_last_error;
    return rc;
  }
  ++p->dispatches;
  return SBB200_OK;
}

int sbb200_health(sbb200_provider_t* p, sbb200_health_t* health, char* last_error,
                  size_t last_error_size) {
  if (!p || !health) return -1;
  std::lock_guard<std::mutex> lock(p->mu);
  std::memset(health, 0, sizeof(*health));
  health->generation = p->generation;
  health->dispatches = p->dispatches;
  health->allocations = p->allocations;
  health->last_error_bytes = p->last_error.size() + 1;
  health->loaded = p->layers.empty() ? 0u : 1u;
  health->pending = 0;
  health->stopped = 0;
  // the device error word of the last forward (bit 0: a kernel wait gave up
  // and its result is not valid); reading it waits for the device
  if (p->dispatches > 0 && p->workspace) {
    int prev = 0;
    cudaGetDevice(&prev);
    uint32_t word = 0;
    cudaError_t e = cudaSetDevice(p->device);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess)
      e = cudaMemcpy(&word, static_cast<const char*>(p->workspace) + sbb::kStatusOffset + 4,
                     sizeof word, cudaMemcpyDeviceToHost);
    cudaSetDevice(prev);
    health->device_errors = e == cudaSuccess ? word : 0x80000000u;
  }
  if (last_error && last_error_size) {
    const size_t need = p->last_error.size() + 1;
    const size_t n = need <= last_error_size ? need - 1 : last_error_size - 1;
    std::memcpy(last_error, p->last_error.data(), n);
    last_error[n] = '\0';
    if (need > last_error_size) return -2;
  }
  return 0;
}

}  // extern "C"
