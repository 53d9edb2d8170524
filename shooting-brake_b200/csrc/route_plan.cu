// Route permutation: histogram of routes per expert, exclusive scan, and a
// STABLE scatter, so the routes of one expert appear in ascending
// route index r = token * top_k + k.
//
// This is the device form of the reference's grouping step
// (src/QuixiCore-XPU/kernels/moe/nvfp4_moe/variants/xpu_sycl/
// nvfp4_moe_grouped.sycl.cpp:140-204: histogram -> scan -> scatter) with the
// order of its CPU tier (src/phase7/cpu_expert_capi.cpp:563-599), where the
// grouped SYCL kernel's atomics would leave the order nondeterministic.
// Ids outside [0, E) are dropped (nvfp4_moe.sycl.cpp:139-141); ids outside
// [-1, E) are also counted into status[0] so the caller can surface them.
//
// Layout: routes are split into chunks of kRouteChunk. Pass 1 writes one
// per-expert count row per chunk. Pass 2 (one CTA per chunk) derives each
// expert's global offset and the chunk's base within the expert from those
// rows, then ranks its routes in order with warp match masks. With a single
// chunk, pass 2 computes the histogram itself and pass 1 is skipped.
#include <atomic>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace sbb {

namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ bool valid_id(int32_t e, int E) { return e >= 0 && e < E; }

// Top-k routing of token t by one warp (the reference's moe_route_topk,
// src/QuixiCore-XPU/kernels/moe/moe_route/variants/xpu_sycl/
// moe_route.sycl.cpp:16-50): k rounds of argmax over the untaken experts with
// a strict '>' (the lowest index wins ties, NaN is never chosen, and a round
// that finds nothing above -inf picks expert 0), then a softmax over the k
// chosen logits, summed in selection order. Lane l holds logits l + 32 j
// (E <= 512); the chosen ids and logits of round i live in lane i % 32.
__device__ void topk_token_warp(const void* __restrict__ logits, int dt, int64_t t, int E, int k,
                                int32_t* ids, float* weights) {
  const int lane = threadIdx.x & 31;
  constexpr int kPer = kMaxExperts / 32;
  float v[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < E ? load_act(logits, static_cast<size_t>(t) * E + e, dt) : 0.0f;
  }
  uint32_t taken = 0;  // bit j: expert lane + 32 j chosen
  int32_t my_sel[2] = {0, 0};
  float my_val[2] = {0.0f, 0.0f};
  for (int i = 0; i < k; ++i) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !((taken >> j) & 1u) && v[j] > best) {
        best = v[j];
        bi = e;
      }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, d);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, d);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (bi == 0x7fffffff) bi = 0;  // nothing above -inf: expert 0, as the reference
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if ((i & 31) == lane) {
      my_sel[i >> 5] = bi;
      my_val[i >> 5] = best;
    }
  }
  // softmax over the chosen logits; max is order-free, the sum follows i
  float m = -INFINITY;
  for (int i = 0; i < k; ++i) m = fmaxf(m, __shfl_sync(0xffffffffu, my_val[i >> 5], i & 31));
  float ex[2] = {0.0f, 0.0f};
  for (int h = 0; h < 2; ++h)
    if (lane + 32 * h < k) ex[h] = expf(my_val[h] - m);
  float sum = 0.0f;
  for (int i = 0; i < k; ++i) sum += __shfl_sync(0xffffffffu, ex[i >> 5], i & 31);
  const float inv = 1.0f / sum;
  for (int h = 0; h < 2; ++h) {
    const int i = lane + 32 * h;
    if (i < k) {
      ids[t * k + i] = my_sel[h];
      weights[t * k + i] = ex[h] * inv;
    }
  }
}

// One token per warp.
__global__ void __launch_bounds__(256) router_topk_kernel(const void* __restrict__ logits, int dt,
                                                          int64_t M, int E, int k,
                                                          int32_t* __restrict__ ids,
                                                          float* __restrict__ weights) {
  pdl_wait();
  pdl_trigger();
  const int64_t t = blockIdx.x * 8ll + (threadIdx.x >> 5);
  if (t < M) topk_token_warp(logits, dt, t, E, k, ids, weights);
}

__global__ void __launch_bounds__(kThreads) route_hist_kernel(
    const int32_t* __restrict__ ids, int64_t R, int E, int32_t* __restrict__ chunk_counts,
    uint32_t* __restrict__ status) {
  extern __shared__ int32_t s_hist[];
  pdl_wait();
  pdl_trigger();
  for (int e = threadIdx.x; e < E; e += kThreads) s_hist[e] = 0;
  __syncthreads();
  const int64_t begin = (int64_t)blockIdx.x * kRouteChunk;
  const int64_t end = min(begin + (int64_t)kRouteChunk, R);
  uint32_t bad = 0;
  for (int64_t r = begin + threadIdx.x; r < end; r += kThreads) {
    const int32_t e = ids[r];
    if (valid_id(e, E)) {
      atomicAdd(&s_hist[e], 1);
    } else if (e != -1) {
      ++bad;
    }
  }
  if (bad) atomicAdd(&status[0], bad);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kThreads)
    chunk_counts[(int64_t)blockIdx.x * E + e] = s_hist[e];
}

// Shared memory: base[E] (chunk base, then running cursor), offs[E + 1],
// warp_cnt[kWarps * E].
// With `logits` (single chunk only) the CTA first routes its tokens itself
// (one warp per token, ids and weights written to `ids`/`weights`), so
// routing from router logits costs no extra launch.
__global__ void __launch_bounds__(kThreads) route_scatter_kernel(
    const int32_t* ids, int64_t R, int E, int nchunks,
    const int32_t* __restrict__ chunk_counts, int32_t* __restrict__ counts,
    int32_t* __restrict__ offsets, int32_t* __restrict__ sorted,
    int32_t* __restrict__ slot_of, uint32_t* __restrict__ status, const void* logits,
    int logits_dt, int top_k, float* weights) {
  extern __shared__ int32_t smem[];
  int32_t* s_base = smem;                // [E]
  int32_t* s_offs = s_base + E;          // [E + 1]
  int32_t* s_wcnt = s_offs + (E + 1);    // [kWarps * E]
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int c = blockIdx.x;
  const int64_t begin = (int64_t)c * kRouteChunk;
  const int64_t end = min(begin + (int64_t)kRouteChunk, R);
  pdl_wait();
  pdl_trigger();
  if (logits) {
    const int64_t M = R / top_k;
    for (int64_t t = warp; t < M; t += kWarps)
      topk_token_warp(logits, logits_dt, t, E, top_k, const_cast<int32_t*>(ids), weights);
    __syncthreads();  // the CTA's own global writes are visible to it after the barrier
  }

  // 1. per-expert totals and this chunk's base.
  if (nchunks == 1) {
    for (int e = tid; e < E; e += kThreads) s_base[e] = 0;
    __syncthreads();
    uint32_t bad = 0;
    for (int64_t r = begin + tid; r < end; r += kThreads) {
      const int32_t e = ids[r];
      if (valid_id(e, E)) atomicAdd(&s_base[e], 1);
      else if (e != -1) ++bad;
    }
    if (bad) atomicAdd(&status[0], bad);
    __syncthreads();
    for (int e = tid; e < E; e += kThreads) {
      s_offs[e + 1] = s_base[e];  // total
      s_base[e] = 0;              // chunk base within the expert
    }
  } else {
    for (int e = tid; e < E; e += kThreads) {
      int32_t before = 0, total = 0;
      for (int cc = 0; cc < nchunks; ++cc) {
        const int32_t v = chunk_counts[(int64_t)cc * E + e];
        before += cc < c ? v : 0;
        total += v;
      }
      s_base[e] = before;
      s_offs[e + 1] = total;
    }
  }
  __syncthreads();
  // 2. exclusive scan of totals (E is small: one warp walks it in 32-wide
  //    steps with a shuffle scan per step).
  if (warp == 0) {
    int32_t carry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      int32_t v = e < E ? s_offs[e + 1] : 0;
      for (int d = 1; d < 32; d <<= 1) {
        const int32_t n = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += n;
      }
      if (e < E) s_offs[e + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) s_offs[0] = 0;
  }
  __syncthreads();
  if (c == 0) {
    for (int e = tid; e < E; e += kThreads) {
      counts[e] = s_offs[e + 1] - s_offs[e];
      offsets[e] = s_offs[e];
    }
    if (tid == 0) offsets[E] = s_offs[E];
  }
  // 3. stable ranks, 1024 routes per step.
  for (int64_t step = begin; step < end; step += kThreads) {
    for (int i = tid; i < kWarps * E; i += kThreads) s_wcnt[i] = 0;
    __syncthreads();
    const int64_t r = step + tid;
    const int32_t e = r < end ? ids[r] : -1;
    const bool ok = r < end && valid_id(e, E);
    const uint32_t active = __ballot_sync(0xffffffffu, ok);
    uint32_t peers = __match_any_sync(0xffffffffu, ok ? e : -1);
    peers &= active;
    const int rank_in_warp = __popc(peers & lanemask_lt());
    if (ok && rank_in_warp == 0) s_wcnt[warp * E + e] = __popc(peers);
    __syncthreads();
    int32_t slot = -1;
    if (ok) {
      int32_t before = 0;
      for (int w = 0; w < warp; ++w) before += s_wcnt[w * E + e];
      slot = s_offs[e] + s_base[e] + before + rank_in_warp;
    }
    __syncthreads();  // every thread has read s_base before it advances
    for (int x = tid; x < E; x += kThreads) {
      int32_t add = 0;
      for (int w = 0; w < kWarps; ++w) add += s_wcnt[w * E + x];
      s_base[x] += add;
    }
    if (r < end) {
      slot_of[r] = slot;
      if (ok) sorted[slot] = (int32_t)r;
    }
    __syncthreads();
  }
}

}  // namespace

size_t route_plan_chunks(int64_t R) { return (size_t)((R + kRouteChunk - 1) / kRouteChunk); }

size_t route_scatter_smem(int E) { return sizeof(int32_t) * ((size_t)E + (E + 1) + (size_t)kWarps * E); }

cudaError_t launch_route_plan(const int32_t* ids, int64_t R, int E, int32_t* chunk_counts,
                              int32_t* counts, int32_t* offsets, int32_t* sorted,
                              int32_t* slot_of, uint32_t* status, cudaStream_t stream,
                              const void* logits, int logits_dt, int top_k, float* weights) {
  const int nchunks = (int)route_plan_chunks(R);
  if (nchunks == 0) {
    // No routes: counts and offsets are all zero.
    cudaError_t err = cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, stream);
    if (err != cudaSuccess) return err;
    return cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (E + 1), stream);
  }
  const size_t smem = route_scatter_smem(E);
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  // once per device; a repeat from a racing thread is harmless
  static std::atomic<bool> attr_set[64] = {};
  if (dev < 0 || dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
    err = cudaFuncSetAttribute(route_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)route_scatter_smem(kMaxExperts));
    if (err != cudaSuccess) return err;
    if (dev >= 0 && dev < 64) attr_set[dev].store(true, std::memory_order_release);
  }
  // the first launch of the plan waits for everything before it; later ones
  // overlap their predecessor's tail
  bool pdl = false;
  const void* fused_logits = nullptr;
  if (logits) {
    if (nchunks == 1) {
      fused_logits = logits;
    } else {
      const int64_t M = R / top_k;
      err = launch_kernel(false, router_topk_kernel, dim3((unsigned)((M + 7) / 8)), dim3(256), 0,
                          stream, logits, logits_dt, M, E, top_k, const_cast<int32_t*>(ids),
                          weights);
      if (err != cudaSuccess) return err;
      pdl = true;
    }
  }
  if (nchunks > 1) {
    err = launch_kernel(pdl, route_hist_kernel, dim3(nchunks), dim3(kThreads),
                        sizeof(int32_t) * E, stream, ids, R, E, chunk_counts, status);
    if (err != cudaSuccess) return err;
    pdl = true;
  }
  return launch_kernel(pdl, route_scatter_kernel, dim3(nchunks), dim3(kThreads), smem, stream,
                       ids, R, E, nchunks, static_cast<const int32_t*>(chunk_counts), counts,
                       offsets, sorted, slot_of, status, fused_logits, logits_dt, top_k, weights);
}

cudaError_t launch_router_topk(const void* logits, int dt, int64_t M, int E, int k, int32_t* ids,
                               float* weights, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  return launch_kernel(false, router_topk_kernel, dim3((unsigned)((M + 7) / 8)), dim3(256), 0,
                       stream, logits, dt, M, E, k, ids, weights);
}

}  // namespace sbb

// ---------------------------------------------------------------------------
// Route plan without any allocation.
//
// Some callers cannot hand the library a workspace: serving engines whose
// device memory belongs to a pooling allocator that forbids allocations
// outside the pool (and whose pool is sized before the model runs), and thin
// FFI bindings (ctypes, cgo, JNI) that hold only the tensors they were given
// and have no device allocator at all. sbb200_route_plan_static serves them
// with scratch that the library owns: the per-chunk expert counts live in the
// file-scope array below, so a call allocates nothing.
//
// The device address of that array is looked up once per device and kept for
// the life of the process. cudaDeviceReset unloads the library's device image,
// so this entry point is not usable after a reset of a device it has run on.
// ---------------------------------------------------------------------------
#include <mutex>
#include <string>

#include "sbb200.h"

namespace sbb {
namespace {

constexpr int64_t kStaticMaxRoutes = 262144;                      // M * top_k
constexpr int kStaticChunks = static_cast<int>(kStaticMaxRoutes / kRouteChunk);  // 64
constexpr int kStaticWords = kStaticChunks * kMaxExperts + 64;     // counts + status

// 128 KB + 256 B on every device that loads the library, held until exit.
// Every call shares it: [0, kStaticChunks * kMaxExperts) per-chunk counts
// (fully rewritten by each multi-chunk call before it is read), then the
// status word that counts out-of-range ids when the caller passes no counter
// (cleared by each such call).
static __device__ __align__(256) int32_t g_route_scratch[kStaticWords];

std::mutex g_route_scratch_mu;
int32_t* g_route_scratch_dev[64] = {};  // device address per device, from set-up

}  // namespace
}  // namespace sbb

extern "C" int sbb200_route_plan_static(void* stream, const int32_t* topk_ids, size_t M,
                                        size_t top_k, size_t E, int32_t* counts,
                                        int32_t* offsets, int32_t* sorted, int32_t* slot_of,
                                        uint32_t* bad_ids) {
  using namespace sbb;
  // M * top_k is formed only once it cannot wrap around
  if (top_k != 0 && M > static_cast<size_t>(kStaticMaxRoutes) / top_k) {
    set_last_error("route_plan_static: M*top_k routes exceed its static scratch limit of "
                   "262144; use sbb200_route_plan with a caller workspace");
    return SBB200_EUNSUPPORTED;
  }
  const size_t R = M * top_k;
  if (E == 0 || E > static_cast<size_t>(kMaxExperts)) {
    set_last_error("route_plan_static: E must be in [1, 512]");
    return SBB200_EINVAL;
  }
  if (R > static_cast<size_t>(kStaticMaxRoutes)) {
    set_last_error("route_plan_static: " + std::to_string(R) +
                   " routes (M*top_k) exceed its static scratch limit of 262144; use "
                   "sbb200_route_plan with a caller workspace");
    return SBB200_EUNSUPPORTED;
  }
  if (!counts || !offsets || (R != 0 && (!topk_ids || !sorted || !slot_of))) {
    set_last_error("route_plan_static received a null pointer");
    return SBB200_EINVAL;
  }
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess || dev < 0 || dev >= 64) {
    set_last_error(std::string("route_plan_static: no usable current device: ") +
                   cudaGetErrorString(err));
    return SBB200_ECUDA;
  }
  int32_t* scratch = nullptr;
  {
    // Set-up, once per device, with that device current: the array's name in
    // host code is only a host-side stand-in, its device address comes from
    // the runtime.
    std::lock_guard<std::mutex> lock(g_route_scratch_mu);
    if (!g_route_scratch_dev[dev]) {
      void* p = nullptr;
      err = cudaGetSymbolAddress(&p, g_route_scratch);
      if (err != cudaSuccess || !p) {
        set_last_error(std::string("route_plan_static: cudaGetSymbolAddress failed: ") +
                       cudaGetErrorString(err));
        return SBB200_ECUDA;
      }
      g_route_scratch_dev[dev] = static_cast<int32_t*>(p);
    }
    scratch = g_route_scratch_dev[dev];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t* status = bad_ids;
  if (!status) {
    status = reinterpret_cast<uint32_t*>(scratch + kStaticChunks * kMaxExperts);
    err = cudaMemsetAsync(status, 0, sizeof(uint32_t), s);
    if (err != cudaSuccess) {
      set_last_error(std::string("route_plan_static: ") + cudaGetErrorString(err));
      return SBB200_ECUDA;
    }
  }
  err = launch_route_plan(topk_ids, static_cast<int64_t>(R), static_cast<int>(E), scratch, counts,
                          offsets, sorted, slot_of, status, s);
  if (err != cudaSuccess) {
    set_last_error(std::string("route_plan_static: ") + cudaGetErrorString(err));
    return SBB200_ECUDA;
  }
  return SBB200_OK;
}
