// Expert parallelism over NVLink: the routed experts of a layer are sharded
// contiguously over the GPUs of one node (one process per GPU), the tokens
// stay with the rank that owns them, and each step exchanges activations and
// per-route outputs through peer memory.
//
// The reference splits experts disjointly over its cards with dense per-card
// slot maps; every card sees all routes with foreign experts as -1 and the
// host sums the per-card partial outputs (src/phase4/src/shooting_brake_vllm/
// routed_experts.py:354-382, 2460-2463, 2522-2524). Here the exchange is
// device-resident and stream-ordered. A step's virtual tokens are
// v = s * max_tokens + t over every source rank s; a destination d serves the
// routes of all virtual tokens that go to its experts.
//
// Decode-sized steps (world * max_tokens * top_k <= 1,024 virtual routes),
// five kernels:
//   exchange split  the CTAs of d's own tokens copy them into d's exchange
//                   buffer and the last of them raises ready[d] = epoch << 32
//                   | M on every rank; every CTA waits for the other ranks'
//                   ready flags, plans d's local routes from every rank's ids
//                   and pulls its token's row from its source GPU
//                   (ep_split_kernel, moe_bs.cu);
//   gate/up, SwiGLU split, down   the single-GPU kernels on d's shard; the
//                   down epilogue stores each route's fp32 row straight into
//                   the source's partial[t][k] (no combine kernel);
//   final  (s)      block 0 raises done[s] = epoch on every rank (s's pushes,
//                   the kernel before, are complete); every block waits for
//                   every rank's done flag and sums its token's routes,
//                   w[t,k] * partial[t][k], in ascending k: the single-GPU
//                   combine's arithmetic and order, so the result does not
//                   depend on how the experts are sharded. The last block
//                   moves the device epoch to the next step.
// Larger steps: a publish kernel, a gather kernel (raises ready, waits,
// keeps the local routes), the route plan, the split pulling rows from the
// sources, the same GEMMs and final.
//
// Flags are raised only after the writes they announce have completed: by
// the kernel after the writing one (griddepcontrol.wait has returned), or,
// inside the exchange split, by the last publishing CTA after every writer
// fenced its stores at system scope. No NCCL call is on the data path; the
// process group only exchanges the CUDA IPC handles of the exchange buffers
// once. The buffers are reused every step without a barrier: a source
// republishes only after its final kernel has seen every rank's done flag
// (raised after that rank's last read of the step), and a destination
// pushes rows for step i+1 only after it saw that source's ready flag for
// step i+1, raised after the source finished reading step i. Every wait
// gives up after 2 s and raises an error bit instead of spinning forever. No
// TMA or bulk copy touches peer memory: peer data moves with plain loads and
// stores.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "moe_driver.h"
#include "sbb200.h"

namespace sbb {
namespace {

constexpr int kEpThreads = 256;

inline size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// Exchange buffer of one rank (identical layout on every rank; peers write
// ready/done flags and per-route rows into it).
struct ExLayout {
  size_t ready;    // u64[world]: ready[s] written by source s
  size_t done;     // u64[world]: done[d] written by destination d
  size_t hidden;   // act [max_tokens, K]
  size_t ids;      // i32 [max_tokens, top_k]
  size_t weights;  // f32 [max_tokens, top_k]
  size_t partial;  // f32 [max_tokens, top_k, K]: row (t, k) written by the
                   // owner of route (t, k)'s expert
  size_t total;
};

ExLayout ex_layout(int world, size_t max_tokens, size_t top_k, size_t K, size_t act_bytes) {
  ExLayout l{};
  size_t at = 0;
  auto take = [&](size_t b) {
    const size_t h = at;
    at = align256(at + b);
    return h;
  };
  l.ready = take(world * 8);
  l.done = take(world * 8);
  l.hidden = take(max_tokens * K * act_bytes);
  l.ids = take(max_tokens * top_k * 4);
  l.weights = take(max_tokens * top_k * 4);
  l.partial = take(max_tokens * top_k * K * 4);
  l.total = at;
  return l;
}

// Copy this step's tokens into the exchange buffer (larger steps).
__global__ void __launch_bounds__(kEpThreads) ep_publish_kernel(
    const uint4* __restrict__ hidden, int64_t hidden_vec, const int32_t* __restrict__ ids,
    const float* __restrict__ weights, int64_t routes, uint4* __restrict__ ex_hidden,
    int32_t* __restrict__ ex_ids, float* __restrict__ ex_weights) {
  pdl_wait();
  pdl_trigger();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden_vec; i += stride)
    ex_hidden[i] = hidden[i];
  for (int64_t i = blockIdx.x * blockDim.x + threadIdx.x; i < routes; i += stride) {
    ex_ids[i] = ids[i];
    ex_weights[i] = weights[i];
  }
}

// Raised by block 0 of the kernel after the one whose writes it announces:
// that kernel has completed and its memory operations are performed
// (griddepcontrol.wait returned, or plain stream order), so a system-scope
// fence and release stores make them visible to every rank before the flags.
__device__ __forceinline__ void raise_flags(unsigned long long* const* at_peer, int world,
                                            int rank, unsigned long long value) {
  if (blockIdx.x != 0 || blockIdx.y != 0) return;
  if (threadIdx.x < world && threadIdx.x != rank) {
    __threadfence_system();
    st_release_sys(at_peer[threadIdx.x], value);
  }
}

// Larger steps: announce this rank's tokens (ready[rank] = epoch << 32 | M on
// every rank), then keep the local routes of every virtual token
// v = s * max_tokens + t.
__global__ void __launch_bounds__(kEpThreads) ep_gather_kernel(
    const unsigned long long* __restrict__ ready, EpDev* dev, const EpTables* __restrict__ tab,
    int world, int64_t max_tokens, int top_k, int rank, int64_t M,
    int32_t* __restrict__ local_ids) {
  __shared__ int64_t s_count[kMaxWorld];
  pdl_wait();
  pdl_trigger();
  const unsigned long long epoch = dev->epoch;
  raise_flags(const_cast<unsigned long long* const*>(tab->ready_at_peer), world, rank,
              (epoch << 32) | static_cast<unsigned long long>(M));
  const uint64_t deadline = globaltimer_ns() + kEpWaitNs;
  for (int s = threadIdx.x; s < world; s += blockDim.x) {
    unsigned long long v = 0;
    if (s == rank) {  // this rank's own tokens: published by the kernel before
      s_count[s] = M;
      continue;
    }
    s_count[s] = ep_wait_epoch(&ready[s], epoch, true, &v, &dev->errors, deadline)
                     ? static_cast<int64_t>(v & 0xffffffffull)
                     : 0;
  }
  __syncthreads();
  const int e_lo = tab->shard_begin[rank];
  const int e_hi = tab->shard_begin[rank + 1];
  const int64_t total = static_cast<int64_t>(world) * max_tokens * top_k;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t v = i / top_k;
    const int s = static_cast<int>(v / max_tokens);
    const int64_t t = v % max_tokens;
    int32_t lid = -1;
    if (t < s_count[s]) {
      const int32_t e = __ldcg(tab->peer_ids[s] + t * top_k + (i % top_k));
      if (e >= e_lo && e < e_hi) lid = e - e_lo;
    }
    local_ids[i] = lid;
  }
}

// out[t] = sum over this token's valid routes k (ascending) of
// w[t, k] * partial[t][k], after every rank's done flag for this step.
__global__ void __launch_bounds__(kEpThreads) ep_final_kernel(
    const unsigned long long* __restrict__ done, EpDev* dev, const EpTables* __restrict__ tab,
    int world, int rank, const int32_t* __restrict__ ids, const float* __restrict__ weights,
    int multiply_router_weight, int top_k, int E, const float* __restrict__ partial, int64_t M,
    int K, void* __restrict__ out, int out_dt) {
  __shared__ int s_k[kMaxTopK];
  __shared__ float s_w[kMaxTopK];
  const int64_t t = blockIdx.x;
  pdl_wait();
  pdl_trigger();
  const unsigned long long epoch = dev->epoch;
  // this rank's pushes (the down projection before this kernel) are in place
  raise_flags(const_cast<unsigned long long* const*>(tab->done_at_peer), world, rank, epoch);
  if (t < M && threadIdx.x < top_k) {
    const int32_t e = ids[t * top_k + threadIdx.x];
    s_k[threadIdx.x] = (e >= 0 && e < E) ? 1 : 0;
    s_w[threadIdx.x] = multiply_router_weight ? weights[t * top_k + threadIdx.x] : 1.0f;
  }
  const uint64_t deadline = globaltimer_ns() + kEpWaitNs;
  for (int d = threadIdx.x; d < world; d += blockDim.x) {
    unsigned long long v = 0;
    if (d != rank)  // this rank's own pushes: the kernel before
      ep_wait_epoch(&done[d], epoch, false, &v, &dev->errors, deadline);
  }
  __syncthreads();
  if (t < M) {
    for (int n4 = (blockIdx.y * blockDim.x + threadIdx.x) * 4; n4 < K;
         n4 += gridDim.y * blockDim.x * 4) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      // routes in groups of 8: the group's loads first, the sums in
      // ascending k
      for (int k0 = 0; k0 < top_k; k0 += 8) {
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          v[j] = (k0 + j < top_k && s_k[k0 + j])
                     ? __ldcg(reinterpret_cast<const float4*>(
                           partial + (t * top_k + k0 + j) * static_cast<int64_t>(K) + n4))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (k0 + j >= top_k || !s_k[k0 + j]) continue;
          const float w = s_w[k0 + j];
          acc.x = fmaf(w, v[j].x, acc.x);
          acc.y = fmaf(w, v[j].y, acc.y);
          acc.z = fmaf(w, v[j].z, acc.z);
          acc.w = fmaf(w, v[j].w, acc.w);
        }
      }
      const int64_t at = t * K + n4;
      if (out_dt == kF32) {
        *reinterpret_cast<float4*>(static_cast<float*>(out) + at) = acc;
      } else if (out_dt == kBF16) {
        __nv_bfloat162 a = __floats2bfloat162_rn(acc.x, acc.y);
        __nv_bfloat162 b = __floats2bfloat162_rn(acc.z, acc.w);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + at) =
            make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
      } else {
        __half2 a = __floats2half2_rn(acc.x, acc.y);
        __half2 b = __floats2half2_rn(acc.z, acc.w);
        *reinterpret_cast<uint2*>(static_cast<__half*>(out) + at) =
            make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
      }
    }
  }
  // every block has read this step's epoch; the last one moves it on
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int total = gridDim.x * gridDim.y;
    if (atomicAdd(&dev->final_count, 1u) + 1u == total) {
      dev->final_count = 0u;
      __threadfence();
      dev->epoch = epoch + 1ull;
    }
  }
}

size_t act_size(int dt) { return dt == SBB200_F32 ? 4 : 2; }

}  // namespace

// Contiguous expert shards: the first E % world ranks hold one extra expert.
void ep_shard(size_t E, int world, int rank, size_t* begin, size_t* count) {
  const size_t base = E / world, extra = E % world;
  const size_t r = static_cast<size_t>(rank);
  *begin = r * base + (r < extra ? r : extra);
  *count = base + (r < extra ? 1 : 0);
}

}  // namespace sbb

struct sbb200_ep {
  int device = 0, rank = 0, world = 1, act_dt = SBB200_BF16, act_terms = sbb::kSplitTerms;
  size_t max_tokens = 0, top_k = 0, E = 0, K = 0, I = 0, e_begin = 0, e_count = 0;
  sbb::ExLayout lay{};
  char* ex = nullptr;                 // this rank's exchange buffer (IPC-exported)
  std::vector<char*> peers;           // opened peer buffers (own buffer at [rank])
  sbb::EpDev* dev = nullptr;          // local device state
  sbb::EpTables* tab = nullptr;       // device copy of the peer tables
  sbb::EpTables host_tab{};
  int32_t* local_ids = nullptr;       // [world * max_tokens, top_k] (larger steps)
  void* workspace = nullptr;          // MoE workspace for world * max_tokens tokens
  bool fused = false;                 // steps exchanged by the activation split
  sbb::WorkspacePlan plan{};
  bool connected = false;
  std::mutex mu;
};

namespace {

int ep_fail(int code, const std::string& msg) {
  sbb::set_last_error(msg);
  return code;
}

struct DeviceGuard {
  int prev = 0;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() { cudaSetDevice(prev); }
};

void ep_free(sbb200_ep* p) {
  DeviceGuard g(p->device);
  for (int i = 0; i < static_cast<int>(p->peers.size()); ++i)
    if (p->peers[i] && i != p->rank) cudaIpcCloseMemHandle(p->peers[i]);
  cudaFree(p->ex);
  cudaFree(p->dev);
  cudaFree(p->tab);
  cudaFree(p->local_ids);
  cudaFree(p->workspace);
}

}  // namespace

extern "C" {

int sbb200_ep_shard(size_t E, int world, int rank, size_t* begin, size_t* count) {
  if (world < 1 || world > sbb::kMaxWorld || rank < 0 || rank >= world || !begin || !count ||
      E < static_cast<size_t>(world))
    return ep_fail(SBB200_EINVAL, "ep shard: need 1 <= world <= 64, 0 <= rank < world, E >= world");
  sbb::ep_shard(E, world, rank, begin, count);
  return SBB200_OK;
}

sbb200_ep_t* sbb200_ep_create(int device, int rank, int world, size_t max_tokens, size_t top_k,
                              size_t E, size_t K, size_t I, int act_dt, int w4a4) {
  try {
    std::string why;
    if (world < 1 || world > sbb::kMaxWorld || rank < 0 || rank >= world) {
      sbb::set_last_error("ep create: need 1 <= world <= 64 and 0 <= rank < world");
      return nullptr;
    }
    if (max_tokens == 0 || E < static_cast<size_t>(world) ||
        sbb::validate_shape(max_tokens * world, E, top_k, K, I, act_dt, SBB200_F32, &why) != 0) {
      sbb::set_last_error("ep create: " + (why.empty() ? std::string("need max_tokens > 0 and E >= world") : why));
      return nullptr;
    }
    if (K % 256 != 0 || I % 256 != 0 || E >= (1u << 31)) {
      sbb::set_last_error("ep create: expert parallelism needs K and I multiples of 256");
      return nullptr;
    }
    auto* p = new (std::nothrow) sbb200_ep();
    if (!p) return nullptr;
    p->device = device;
    p->rank = rank;
    p->world = world;
    p->act_dt = act_dt;
    p->act_terms = w4a4 ? 1 : sbb::kSplitTerms;
    p->max_tokens = max_tokens;
    p->top_k = top_k;
    p->E = E;
    p->K = K;
    p->I = I;
    sbb::ep_shard(E, world, rank, &p->e_begin, &p->e_count);
    p->lay = sbb::ex_layout(world, max_tokens, top_k, K, sbb::act_size(act_dt));
    const size_t vt = static_cast<size_t>(world) * max_tokens;
    const size_t e_local_max = (E + world - 1) / world;
    p->plan = sbb::plan_workspace(vt, e_local_max, top_k, K, I);
    p->fused = sbb::ep_split_fits(static_cast<int64_t>(vt), static_cast<int>(top_k),
                                  static_cast<int>(K), static_cast<int>(I),
                                  static_cast<int>(e_local_max));
    DeviceGuard g(device);
    cudaError_t e = g.ok ? cudaSuccess : cudaErrorInvalidDevice;
    if (e == cudaSuccess) e = cudaMalloc(&p->ex, p->lay.total);
    if (e == cudaSuccess) e = cudaMemset(p->ex, 0, p->lay.hidden);  // ready and done flags
    if (e == cudaSuccess) e = cudaMalloc(&p->dev, sizeof(sbb::EpDev));
    // epochs start at 1, so the zeroed flags match no step
    sbb::EpDev init{};
    init.epoch = 1ull;
    if (e == cudaSuccess) e = cudaMemcpy(p->dev, &init, sizeof init, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&p->tab, sizeof(sbb::EpTables));
    if (e == cudaSuccess && !p->fused) e = cudaMalloc(&p->local_ids, vt * top_k * 4);
    if (e == cudaSuccess) e = cudaMalloc(&p->workspace, p->plan.total);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      sbb::set_last_error(std::string("ep create: ") + cudaGetErrorString(e));
      ep_free(p);
      delete p;
      return nullptr;
    }
    return p;
  } catch (...) {
    sbb::set_last_error("ep create: host exception");
    return nullptr;
  }
}

int sbb200_ep_ipc_handle(sbb200_ep_t* p, void* out, size_t size) {
  if (!p || !out || size < sizeof(cudaIpcMemHandle_t))
    return ep_fail(SBB200_EINVAL, "ep handle: null handle or buffer below SBB200_EP_HANDLE_BYTES");
  DeviceGuard g(p->device);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, p->ex);
  if (e != cudaSuccess) return ep_fail(SBB200_ECUDA, std::string("ep handle: ") + cudaGetErrorString(e));
  std::memcpy(out, &h, sizeof h);
  return SBB200_OK;
}

int sbb200_ep_connect(sbb200_ep_t* p, const void* handles, size_t size) {
  if (!p || !handles || size < sizeof(cudaIpcMemHandle_t) * p->world)
    return ep_fail(SBB200_EINVAL, "ep connect: need world * SBB200_EP_HANDLE_BYTES handle bytes");
  std::lock_guard<std::mutex> lk(p->mu);
  if (p->connected) return ep_fail(SBB200_EINVAL, "ep connect: already connected");
  DeviceGuard g(p->device);
  p->peers.assign(p->world, nullptr);
  for (int r = 0; r < p->world; ++r) {
    if (r == p->rank) {
      p->peers[r] = p->ex;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const char*>(handles) + r * sizeof h, sizeof h);
    void* ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int i = 0; i < r; ++i)
        if (i != p->rank && p->peers[i]) cudaIpcCloseMemHandle(p->peers[i]);
      p->peers.assign(p->world, nullptr);
      return ep_fail(SBB200_ECUDA, "ep connect: opening the buffer of rank " + std::to_string(r) +
                                       ": " + cudaGetErrorString(e));
    }
    p->peers[r] = static_cast<char*>(ptr);
  }
  sbb::EpTables& t = p->host_tab;
  std::memset(&t, 0, sizeof t);
  for (int r = 0; r < p->world; ++r) {
    char* b = p->peers[r];
    t.ready_at_peer[r] = reinterpret_cast<unsigned long long*>(b + p->lay.ready) + p->rank;
    t.done_at_peer[r] = reinterpret_cast<unsigned long long*>(b + p->lay.done) + p->rank;
    t.peer_hidden[r] = b + p->lay.hidden;
    t.peer_ids[r] = reinterpret_cast<const int32_t*>(b + p->lay.ids);
    t.peer_weights[r] = reinterpret_cast<const float*>(b + p->lay.weights);
    t.partial_at_peer[r] = reinterpret_cast<float*>(b + p->lay.partial);
  }
  for (int r = 0; r <= p->world; ++r) {
    size_t b = 0, c = 0;
    if (r < p->world) {
      sbb::ep_shard(p->E, p->world, r, &b, &c);
    } else {
      b = p->E;
    }
    t.shard_begin[r] = static_cast<int>(b);
  }
  const cudaError_t e = cudaMemcpy(p->tab, &t, sizeof t, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return ep_fail(SBB200_ECUDA, std::string("ep connect: ") + cudaGetErrorString(e));
  p->connected = true;
  return SBB200_OK;
}

int sbb200_ep_forward_staged(sbb200_ep_t* p, void* stream, const void* hidden,
                             const int32_t* topk_ids, const float* topk_weights, size_t M,
                             const void* w13, const void* w13_scales,
                             const float* w13_global_scales, const void* w2,
                             const void* w2_scales, const float* w2_global_scales, void* out,
                             int out_dt, int multiply_router_weight, void* const* stage_events,
                             size_t n_stage_events) {
  try {
    if (stage_events && n_stage_events < SBB200_EP_STAGE_EVENTS)
      return ep_fail(SBB200_EINVAL, "ep forward: need SBB200_EP_STAGE_EVENTS stage events");
    if (!p) return ep_fail(SBB200_EINVAL, "ep forward: null handle");
    if (!p->connected) return ep_fail(SBB200_EINVAL, "ep forward: connect the ranks first");
    if (M > p->max_tokens)
      return ep_fail(SBB200_EINVAL, "ep forward: M above the max_tokens given at create");
    if ((M && (!hidden || !topk_ids || !topk_weights || !out)) || !w13 || !w13_scales ||
        !w13_global_scales || !w2 || !w2_scales || !w2_global_scales)
      return ep_fail(SBB200_EINVAL, "ep forward: null pointer argument");
    if (out_dt != SBB200_F32 && out_dt != SBB200_F16 && out_dt != SBB200_BF16)
      return ep_fail(SBB200_EINVAL, "ep forward: output dtype must be f32, f16 or bf16");
    if ((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(out)) % 16 != 0)
      return ep_fail(SBB200_EINVAL, "ep forward: hidden and out must be 16-byte aligned");
    std::lock_guard<std::mutex> lk(p->mu);
    DeviceGuard g(p->device);
    auto s = static_cast<cudaStream_t>(stream);
    auto mark = [&](int i) {
      if (stage_events && stage_events[i])
        sbb::record_stage_event(static_cast<cudaEvent_t>(stage_events[i]), s);
    };
    mark(0);
    const int64_t K = static_cast<int64_t>(p->K);
    const int64_t routes = static_cast<int64_t>(M * p->top_k);
    const int64_t vt = static_cast<int64_t>(p->world) * p->max_tokens;
    char* ex = p->ex;
    char* tab = reinterpret_cast<char*>(p->tab);  // device address, not dereferenced here
    sbb::EpSplitArgs xa{};
    if (p->fused) {
      // the activation split publishes, announces and gathers the step itself
      xa.tab = p->tab;
      xa.dev = p->dev;
      xa.ready = reinterpret_cast<const unsigned long long*>(ex + p->lay.ready);
      xa.hidden = hidden;
      xa.ids = topk_ids;
      xa.weights = topk_weights;
      xa.ex_hidden = ex + p->lay.hidden;
      xa.ex_ids = reinterpret_cast<int32_t*>(ex + p->lay.ids);
      xa.ex_weights = reinterpret_cast<float*>(ex + p->lay.weights);
      xa.world = p->world;
      xa.rank = p->rank;
      xa.act_bytes = static_cast<int>(sbb::act_size(p->act_dt));
      xa.M = static_cast<int64_t>(M);
      xa.max_tokens = static_cast<int64_t>(p->max_tokens);
      mark(1);
      mark(2);
    } else {
      // 1. publish
      const int64_t vec = static_cast<int64_t>(M) * K * sbb::act_size(p->act_dt) / 16;
      int blocks = static_cast<int>(
          std::min<int64_t>(148 * 4, (vec + sbb::kEpThreads - 1) / sbb::kEpThreads));
      if (blocks < 1) blocks = 1;
      cudaError_t e = sbb::launch_kernel(
          true, sbb::ep_publish_kernel, dim3(blocks), dim3(sbb::kEpThreads), 0, s,
          static_cast<const uint4*>(hidden), vec, topk_ids, topk_weights, routes,
          reinterpret_cast<uint4*>(ex + p->lay.hidden), reinterpret_cast<int32_t*>(ex + p->lay.ids),
          reinterpret_cast<float*>(ex + p->lay.weights));
      if (e != cudaSuccess) return ep_fail(SBB200_ECUDA, std::string("ep publish: ") + cudaGetErrorString(e));
      mark(1);
      // 2. gather the local routes of every source
      const int64_t total = vt * p->top_k;
      blocks = static_cast<int>(
          std::min<int64_t>(148 * 2, (total + sbb::kEpThreads - 1) / sbb::kEpThreads));
      e = sbb::launch_kernel(true, sbb::ep_gather_kernel, dim3(blocks), dim3(sbb::kEpThreads), 0,
                             s, reinterpret_cast<const unsigned long long*>(ex + p->lay.ready),
                             p->dev, static_cast<const sbb::EpTables*>(p->tab), p->world,
                             static_cast<int64_t>(p->max_tokens), static_cast<int>(p->top_k),
                             p->rank, static_cast<int64_t>(M), p->local_ids);
      if (e != cudaSuccess) return ep_fail(SBB200_ECUDA, std::string("ep gather: ") + cudaGetErrorString(e));
      mark(2);
    }
    // 3. the shard's MoE on the virtual tokens: rows pulled from their
    // sources, each route's row pushed back to its source
    {
      sbb::MoeArgs a{};
      a.hidden = nullptr;
      a.act_dt = p->act_dt;
      a.ids = p->local_ids;
      a.weights = nullptr;  // router weights are applied by the source's final sum
      a.multiply_router_weight = multiply_router_weight;
      a.w13 = static_cast<const uint8_t*>(w13);
      a.s13 = static_cast<const uint8_t*>(w13_scales);
      a.g13 = w13_global_scales;
      a.w2 = static_cast<const uint8_t*>(w2);
      a.s2 = static_cast<const uint8_t*>(w2_scales);
      a.g2 = w2_global_scales;
      a.out = nullptr;
      a.out_dt = SBB200_F32;
      a.act_terms = p->act_terms;
      a.M = vt;
      a.E = static_cast<int>(p->e_count);
      a.top_k = static_cast<int>(p->top_k);
      a.K = static_cast<int>(p->K);
      a.I = static_cast<int>(p->I);
      // the expert step's own marks land in events [2..6]: [3] after the
      // split (exchange, route plan), [4] after gate/up, [5] after down
      // (including the pushes), [6] = [5] (no combine)
      a.stage_events = stage_events ? stage_events + 2 : nullptr;
      if (p->fused) {
        a.ep_split = &xa;
      } else {
        a.hidden_rows = sbb::SplitRows{
            reinterpret_cast<const void* const*>(tab + offsetof(sbb::EpTables, peer_hidden)),
            static_cast<int64_t>(p->max_tokens)};
      }
      a.push = sbb::PushRows{
          reinterpret_cast<float* const*>(tab + offsetof(sbb::EpTables, partial_at_peer)),
          static_cast<int64_t>(p->max_tokens)};
      std::string why;
      const cudaError_t e = sbb::run_moe(a, p->plan, p->workspace, s, &why);
      if (e != cudaSuccess) return ep_fail(SBB200_ECUDA, "ep expert step (" + why + "): " + cudaGetErrorString(e));
    }
    // 4. sum the routes of this rank's tokens (with no tokens here the kernel
    // still raises and consumes the done flags, so the exchange stays in step)
    const dim3 grid(M > 0 ? static_cast<unsigned>(M) : 1u,
                    static_cast<unsigned>((K + 4 * sbb::kEpThreads - 1) / (4 * sbb::kEpThreads)));
    const cudaError_t e = sbb::launch_kernel(
        true, sbb::ep_final_kernel, grid, dim3(sbb::kEpThreads), 0, s,
        reinterpret_cast<const unsigned long long*>(ex + p->lay.done), p->dev,
        static_cast<const sbb::EpTables*>(p->tab), p->world, p->rank, topk_ids, topk_weights,
        multiply_router_weight, static_cast<int>(p->top_k), static_cast<int>(p->E),
        reinterpret_cast<const float*>(ex + p->lay.partial), static_cast<int64_t>(M),
        static_cast<int>(K), out, out_dt);
    if (e != cudaSuccess) return ep_fail(SBB200_ECUDA, std::string("ep final: ") + cudaGetErrorString(e));
    mark(7);
    return SBB200_OK;
  } catch (...) {
    return ep_fail(SBB200_ECUDA, "ep forward: host exception");
  }
}

int sbb200_ep_forward(sbb200_ep_t* p, void* stream, const void* hidden, const int32_t* topk_ids,
                      const float* topk_weights, size_t M, const void* w13, const void* w13_scales,
                      const float* w13_global_scales, const void* w2, const void* w2_scales,
                      const float* w2_global_scales, void* out, int out_dt,
                      int multiply_router_weight) {
  return sbb200_ep_forward_staged(p, stream, hidden, topk_ids, topk_weights, M, w13, w13_scales,
                                  w13_global_scales, w2, w2_scales, w2_global_scales, out, out_dt,
                                  multiply_router_weight, nullptr, SBB200_EP_STAGE_EVENTS);
}

int sbb200_ep_launches(const sbb200_ep_t* p) {
  if (!p) return -1;
  // exchange split, gate/up, SwiGLU split, down (pushing), final; larger
  // steps: publish, gather, route plan (1 or 2), split, gate/up, SwiGLU
  // split, down, final. No combine kernel either way.
  if (p->fused) return 5;
  const int64_t vt = static_cast<int64_t>(p->world) * p->max_tokens;
  return 2 + sbb::count_launches(vt, static_cast<int>(p->top_k), static_cast<int>(p->K),
                                 static_cast<int>(p->I), false) - 1 + 1;
}

int sbb200_ep_device_errors(sbb200_ep_t* p, void* stream, uint32_t* errors) {
  if (!p || !errors) return ep_fail(SBB200_EINVAL, "ep errors: null argument");
  DeviceGuard g(p->device);
  auto s = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  char* errs = reinterpret_cast<char*>(p->dev) + offsetof(sbb::EpDev, errors);
  cudaError_t e = cudaMemcpyAsync(&v, errs, 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(errs, 0, 4, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return ep_fail(SBB200_ECUDA, std::string("ep errors: ") + cudaGetErrorString(e));
  *errors = v;
  return SBB200_OK;
}

void sbb200_ep_destroy(sbb200_ep_t* p) {
  if (!p) return;
  ep_free(p);
  delete p;
}

}  // extern "C"
